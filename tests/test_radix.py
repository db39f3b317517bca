"""The library's prefix index (specdec_radix_*, path-compressed) against the
reference's RadixKVCache (server/radix_kv_cache.cpp:39-98).

  * golden: the reference class itself, run by tests/golden/gen_radix_golden.py
    over a 160-call script of inserts and releases with 24 probe matches after
    every call -- the library and the oracle's per-token trie reproduce every
    (matched, source) pair;
  * random scripts (more tokens, longer prompts, many requests): the library
    equals the oracle trie on every probe after every call, and the token
    positions it holds equal the trie's node count (no leaked or missing
    positions after splits and removals).
"""
import os

import numpy as np
import pytest

import radix as RO
import specdec as S

HERE = os.path.dirname(os.path.abspath(__file__))


def _unpack(off, flat):
    return [flat[off[i]:off[i + 1]].tolist() for i in range(len(off) - 1)]


def test_radix_matches_reference_golden():
    g = np.load(os.path.join(HERE, "golden", "radix_golden.npz"))
    ops = list(zip(g["op_kind"].tolist(), g["op_req"].tolist(), _unpack(g["op_off"], g["op_toks"])))
    probes = _unpack(g["probe_off"], g["probe_toks"])
    lib, orc = S.RadixKVCache(), RO.RadixTrie()
    for i, (kind, req, toks) in enumerate(ops):
        for c in (lib, orc):
            c.insert_prefix(req, toks) if kind == 0 else c.release_prefix(req)
        for j, p in enumerate(probes):
            want = tuple(g["results"][i, j].tolist())
            assert lib.match_prefix(p) == want, (i, j)
            assert orc.match_prefix(p) == want, (i, j)
    lib.close()


@pytest.mark.parametrize("seed", range(6))
def test_radix_random_scripts_match_oracle(seed):
    rng = np.random.default_rng(seed)
    V = [3, 8, 50][seed % 3]
    bases = [rng.integers(0, V, 300).tolist() for _ in range(5)]

    def prompt():
        b = bases[int(rng.integers(0, 5))]
        return b[:int(rng.integers(0, 300))] + rng.integers(0, V, int(rng.integers(0, 20))).tolist()

    lib, orc = S.RadixKVCache(), RO.RadixTrie()
    live = []
    for step in range(300):
        u = rng.random()
        if u < 0.5 or not live:
            req, toks = int(rng.integers(0, 40)), prompt()
            lib.insert_prefix(req, toks)
            orc.insert_prefix(req, toks)
            live.append(req)
        else:
            req = live.pop(int(rng.integers(0, len(live)))) if u < 0.95 else 1000 + step
            lib.release_prefix(req)
            orc.release_prefix(req)
        for _ in range(4):
            p = prompt()
            assert lib.match_prefix(p) == orc.match_prefix(p), step
        assert lib.stats()[1] == orc.positions(), step
    lib.close()
