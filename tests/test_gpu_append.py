"""GPU parity of the cache-append kernel (``sqa_cache_append``) against the CPU oracle.

A copy, so the bar is bit-exact: every cache byte after the GPU append equals the
oracle's (``oracle/cache_append.py``), untouched slots included.  Append-then-attend
on the GPU reproduces the golden outputs of the upstream reference.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cache_append_reference
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu

GOLDEN = [p for p in sorted((Path(__file__).parent / "golden").glob("*.npz")) if not p.stem.startswith("upstream_")]


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m

    return m


def _case(seed, batch, q_len, lens, hkv, extra_pages=5):
    rng = np.random.default_rng(seed)
    pages = [(n + 15) // 16 for n in lens]
    pool = sum(pages) + extra_pages
    ids = rng.permutation(pool).astype(np.int32)
    width = max(pages) + 2
    table = np.full((batch, width), pool - 1, np.int32)
    cur = 0
    for b, n in enumerate(pages):
        table[b, :n] = ids[cur:cur + n]
        cur += n
    kc = rng.standard_normal((pool, 16, hkv, 128)).astype(np.float16)
    vc = rng.standard_normal((pool, 16, hkv, 128)).astype(np.float16)
    nk = rng.standard_normal((batch, q_len, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((batch, q_len, hkv, 128)).astype(np.float16)
    return nk, nv, kc, vc, table, np.array(lens, np.int32)


def _cuda(*xs):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in xs]


@pytest.mark.parametrize("q_len,lens,hkv", [
    (1, [1, 16, 17, 1000], 8),
    (2, [2, 15, 16, 33, 4096], 8),
    (4, [4, 20, 64, 65], 2),
    (8, [8, 9, 100, 129, 8192], 8),
    (16, [16, 31, 32, 47, 300], 4),
    (3, [3] * 40 + [777], 1),
])
def test_append_bit_exact(sqa, q_len, lens, hkv):
    nk, nv, kc, vc, table, lens_np = _case(q_len * 7 + len(lens), len(lens), q_len, lens, hkv)
    ek, ev = cache_append_reference(nk, nv, kc, vc, table, lens_np)
    g = _cuda(nk, nv, kc, vc, table, lens_np)
    sqa.cache_append(*g, check=True)
    assert torch.equal(g[2].cpu().view(torch.int16), torch.from_numpy(ek).view(torch.int16))
    assert torch.equal(g[3].cpu().view(torch.int16), torch.from_numpy(ev).view(torch.int16))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_append_then_attend_reproduces_golden(sqa, path):
    """Blank the newest q_len tokens of the golden caches, append them on the GPU,
    then attend on the GPU: the upstream reference's golden output comes back."""
    with np.load(path) as z:
        c = {k: z[k] for k in z.files}
    q_len = c["query"].shape[1]
    kc, vc, table, lens = c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"]
    nk = np.zeros((len(lens), q_len) + kc.shape[2:], kc.dtype)
    nv = np.zeros_like(nk)
    kb, vb = kc.copy(), vc.copy()
    for b, n in enumerate(lens):
        for qi in range(q_len):
            t = int(n) - q_len + qi
            nk[b, qi], nv[b, qi] = kc[table[b, t // 16], t % 16], vc[table[b, t // 16], t % 16]
            kb[table[b, t // 16], t % 16] = np.nan
            vb[table[b, t // 16], t % 16] = np.nan
    q, k, v, t_, l_, n_k, n_v = _cuda(c["query"], kb, vb, table, lens, nk, nv)
    sqa.cache_append(n_k, n_v, k, v, t_, l_, check=True)
    out = sqa.small_q_attention(q, k, v, t_, l_, 16, check=True)
    assert_close(out, c["expected"])


def test_append_errors_are_reported_and_skipped(sqa):
    nk, nv, kc, vc, table, lens = _case(5, 3, 4, [40, 50, 60], 2)
    for bad_lens, exc in (([40, 3, 60], ValueError), ([40, 50, 16 * table.shape[1] + 1], ValueError)):
        lens_np = np.array(bad_lens, np.int32)
        g = _cuda(nk, nv, kc, vc, table, lens_np)
        with pytest.raises(exc):
            sqa.cache_append(*g, check=True)
        # the valid sequences were still written, exactly as the oracle writes them
        ok = [i for i in range(3) if 4 <= bad_lens[i] <= 16 * table.shape[1]]
        ek, _ = cache_append_reference(nk[ok], nv[ok], kc, vc, table[ok], lens_np[ok])
        assert torch.equal(g[2].cpu().view(torch.int16), torch.from_numpy(ek).view(torch.int16))
    bad_table = table.copy()
    bad_table[1, 3] = kc.shape[0] + 3  # the page holding tokens 48..63 of sequence 1 (its newest)
    g = _cuda(nk, nv, kc, vc, bad_table, lens)
    with pytest.raises(IndexError):
        sqa.cache_append(*g, check=True)


def test_append_contract_errors(sqa):
    nk, nv, kc, vc, table, lens = _case(1, 2, 2, [20, 30], 2)
    g = _cuda(nk, nv, kc, vc, table, lens)
    with pytest.raises(ValueError):
        sqa.cache_append(g[0].float(), g[1], g[2], g[3], g[4], g[5])
    with pytest.raises(ValueError):
        sqa.cache_append(g[0], g[1], g[2][:, :8].contiguous(), g[3][:, :8].contiguous(), g[4], g[5])
    with pytest.raises(ValueError):
        sqa.cache_append(g[0], g[1], g[2], g[3], g[4], g[5].long())
