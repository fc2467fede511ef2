"""CPU oracle for the cache-append step (test infrastructure only).

Imported only by ``tests/`` and ``__graft_entry__.smoke()``; the product
package never imports it.

The upstream attention takes ``seq_lens`` as the length after the draft
tokens were appended (``src/small_q_attention/reference.py:25``) and reads
token ``t`` of sequence ``b`` from page ``block_tables[b, t // page_size]``,
slot ``t % page_size`` (``reference.py:54-59``; element layout
``csrc/small_q_attention_ext.cu:466``).  The append that produces such a cache
is restated here: token ``qi`` of the ``q_len`` new tokens is position
``seq_lens[b] - q_len + qi``.  Metadata errors raise what the upstream
reference raises for the same metadata in the attention (``ValueError`` for
``seq_lens < q_len``, ``reference.py:52-53``; ``IndexError`` for a page id
outside the cache, as ``index_select`` does).
"""

from __future__ import annotations

import numpy as np

__all__ = ["cache_append_reference"]


def _np(x):
    if hasattr(x, "detach"):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def cache_append_reference(new_keys, new_values, key_cache, value_cache, block_tables, seq_lens,
                           page_size: int = 16):
    """Return copies of the caches with the new tokens written in."""
    nk, nv = _np(new_keys), _np(new_values)
    kc, vc = _np(key_cache).copy(), _np(value_cache).copy()
    table, lens = _np(block_tables), _np(seq_lens)
    batch, q_len = nk.shape[:2]
    for b in range(batch):
        total = int(lens[b])
        if total < q_len:
            raise ValueError("seq_lens must be at least q_len for MTP attention")
        if (total + page_size - 1) // page_size > table.shape[1]:
            raise ValueError("seq_lens exceeds page_size * block_tables.shape[1]")
        for qi in range(q_len):
            t = total - q_len + qi
            page = int(table[b, t // page_size])
            if not 0 <= page < kc.shape[0]:
                raise IndexError("block_tables holds a page id outside the cache")
            kc[page, t % page_size] = nk[b, qi]
            vc[page, t % page_size] = nv[b, qi]
    return kc, vc
