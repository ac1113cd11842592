"""TEST INFRASTRUCTURE ONLY: the CPU oracle for packed variable-length attention.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this package, and only as the checker or as the timed CPU baseline. The product
package ``packed_encoders_b200`` never imports it; it has no CPU fallback.
"""

from oracle.oracle import (  # noqa: F401
    attention,
    attention_prefixed,
    available_reference,
    build,
    reference_local_attention,
    rope_bshd,
    useful_pairs,
)
