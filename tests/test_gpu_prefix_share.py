"""Prefix sharing in the step engine: specdec_engine_admit with a prefix
index (RadixKVCache semantics, server/radix_kv_cache.cpp:39-98) shares the
KV blocks of an indexed prefix between sequences (PagedKVCache::share_prefix,
server/paged_kv_cache.cpp:136-154) and prefills only the rest.

Checked on the tiny model:
  * shared whole blocks: the tables of the sharing slots start with the
    source's blocks, whose reference counts count every holder, and the pool
    holds fewer blocks than the same admissions without the index;
  * the admitted state equals an engine that prefilled every prompt in full
    (pending tokens equal; draft hidden states and the recomputed KV rows
    within the step-engine tolerance);
  * speculative steps afterwards are in parity with the oracle, as in the
    step-engine test (decisions bit-exact, logits within 2e-2);
  * retiring the source keeps the shared blocks alive for the other holders;
    a prefix whose creating request has retired is not shared (the
    reference's source rule), one created by a live request is.
"""
import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import steps_match_oracle

pytestmark = pytest.mark.gpu

TINY = S.MODEL_SHAPES["tiny"]
CFG = dict(TINY, block_size=16, rms_eps=1e-5, rope_theta=10000.0)


def _kv_rows(eng, b, n):
    """K/V of the first n tokens of slot b: [L, n, 2, Hkv, hd] fp16 values."""
    L, Hkv, hd = TINY["layers"], TINY["n_kv_heads"], TINY["head_dim"]
    nb, mb = eng.info("num_blocks"), eng.info("max_blocks")
    pool = eng.read("kv", np.uint16, (L, nb, 2, Hkv, 16, hd))
    tab = eng.read("tables", np.int32, (eng.batch, mb))[b]
    t = np.arange(n)
    rows = pool[:, tab[t // 16], :, :, t % 16, :]  # [n, L, 2, Hkv, hd] (advanced indices first)
    return O.f16_vals(np.moveaxis(rows, 0, 1))


def test_admit_shares_prefix_blocks(cuda_device):
    B, k, T, seed = 4, 3, 1.0, 7
    V, H = TINY["vocab"], TINY["hidden"]
    rng = np.random.default_rng(11)
    p0 = rng.integers(0, V, 200).astype(np.int32)
    p1 = np.concatenate([p0[:150], rng.integers(0, V, 60)]).astype(np.int32)
    p2 = p0.copy()
    p3 = np.concatenate([p1[:180], rng.integers(0, V, 21)]).astype(np.int32)
    prompts = [p0, p1, p2, p3]
    kw = dict(batch=B, draft_len=k, max_ctx=512, temperature=T, seed=seed, use_graph=True)
    eng, ref = S.Engine(TINY, **kw), S.Engine(TINY, **kw)
    eng.init_weights(0)
    ref.init_weights(0)
    cache = S.RadixKVCache()
    shared = [eng.admit(b, 100 + b, prompts[b], cache) for b in range(B)]
    # p1 shares 150 tokens of p0 -> 144 (whole blocks); p2 = p0 shares its 199 KV
    # tokens up to P - 2 = 198 -> 192; p3 matches 180 tokens of p1, created by
    # request 101 -> 176
    assert shared == [0, 144, 192, 176]
    for b in range(B):
        assert ref.admit(b, 200 + b, prompts[b]) == 0
    mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
    tab = eng.read("tables", np.int32, (B, mb))
    assert tab[1, :9].tolist() == tab[0, :9].tolist()
    assert tab[2, :12].tolist() == tab[0, :12].tolist()
    assert tab[3, :11].tolist() == tab[1, :11].tolist()
    ref_counts = eng.read("refcounts", np.int32, (nb,))
    assert [int(ref_counts[x]) for x in tab[0, :12]] == [4] * 9 + [2] * 3
    assert int(ref_counts[tab[1, 9]]) == 2 and int(ref_counts[tab[1, 10]]) == 2  # p1's blocks 9, 10 shared with p3
    lens = eng.read("lens", np.int32, (B,))
    assert lens.tolist() == [len(p) - 1 for p in prompts] == ref.read("lens", np.int32, (B,)).tolist()
    used = lambda e: int((e.read("refcounts", np.int32, (nb,)) > 0).sum())  # noqa: E731
    assert used(eng) == used(ref) - (9 + 12 + 11)
    # the admitted state equals full prefills
    assert eng.read("pending", np.int32, (B,)).tolist() == ref.read("pending", np.int32, (B,)).tolist()
    h, hr = eng.read("h0", np.float32, (B, H)), ref.read("h0", np.float32, (B, H))
    np.testing.assert_allclose(h, hr, rtol=2e-2, atol=2e-2 * float(np.abs(hr).max()))
    for b in range(B):
        np.testing.assert_allclose(_kv_rows(eng, b, len(prompts[b]) - 1), _kv_rows(ref, b, len(prompts[b]) - 1),
                                   rtol=2e-2, atol=2e-2)
    # speculative steps over the shared blocks, in parity with the oracle
    model = O.OracleModel(CFG, seed=0, rope_max_pos=512 + 80)
    steps_match_oracle(eng, model, TINY, B, k, T, seed, steps=3)
    # the shared prefix blocks never changed
    tab2 = eng.read("tables", np.int32, (B, mb))
    assert tab2[1, :9].tolist() == tab[0, :9].tolist() and tab2[2, :12].tolist() == tab[0, :12].tolist()
    # retire the source: its private blocks go, the shared ones stay with the holders
    eng.retire(0, cache)
    ref_counts = eng.read("refcounts", np.int32, (nb,))
    assert [int(ref_counts[x]) for x in tab[0, :12]] == [3] * 9 + [1] * 3
    # p0 again: its deepest indexed position was created by retired request 100 -> not shared
    assert eng.admit(0, 104, p0, cache) == 0
    # a prompt under p1's prefix, whose creator (101) is live -> shared
    eng.retire(3, cache)
    assert eng.admit(3, 105, np.concatenate([p1[:170], rng.integers(0, V, 5)]).astype(np.int32), cache) == 160
    eng.close()
    ref.close()
    model.close()
    cache.close()
