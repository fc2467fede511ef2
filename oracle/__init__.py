"""CPU oracle for the small-q paged attention path (test infrastructure only).

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py``; the product package never imports it.
"""

from .cache_append import cache_append_reference  # noqa: F401
from .paged_mtp_attention import (  # noqa: F401
    merge_partials,
    paged_mtp_attention_partial,
    paged_mtp_attention_reference,
)
