"""CPU oracle for the paged-KV attention path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker or as the timed
CPU baseline. The product path (``hayate_b200``) never imports it.
"""

from .paged_oracle import (  # noqa: F401
    attention_flops,
    decode_bytes,
    kv_scatter,
    paged_attention,
    scatter_positions,
)
