"""CPU oracle for the two hot paths (test infrastructure, never the product).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference leg may import this package, and only as the checker or the timed CPU
baseline. The CUDA product path never routes through it.
"""

from oracle.oracle import (  # noqa: F401
    decode_bytes,
    fused_add_rms_norm,
    paged_decode_attention,
    rms_norm,
    round_to,
)
