"""CPU check that the vocabulary-sharded acceptance loses nothing: row
statistics assembled from per-shard partials -- the rank-order arg-max
merge, integer mass sums, the top-p threshold from summed per-shard digit
histograms, and the draw as the best of the shards' local winners (race
keys) -- equal the oracle's statistics and draw on the whole row.  These are the
combinations specdec.dist.accept_chain_vocab_sharded performs between the
specdec_shard_* steps; the device kernels themselves are checked against
the oracle in the GPU tests."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from specdec.dist import vocab_shard


def _key(z):
    b = z.astype(np.float32).view(np.uint32).astype(np.uint64)
    return np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000).astype(np.uint64)


def _masses(z, mx, temperature):
    """Integer masses E_j at the row max mx (the oracle's own formula)."""
    st = O.RowStats()
    st.max = float(mx)
    st.tau = 0
    c = O.temp_coeff(temperature)
    zc = np.ascontiguousarray(z, dtype=np.float32)
    return np.array([O.lib().orc_row_mass(O.ptr(zc), C.byref(st), c, j) for j in range(zc.size)], dtype=np.uint64)


def _select(hist, thr, G):
    """Highest digit whose mass from the top reaches thr (select_digit)."""
    cum = G
    for b in range(255, -1, -1):
        if cum + int(hist[b]) >= thr:
            return b, cum, int(hist[b])
        cum += int(hist[b])
    raise AssertionError("threshold above the total")


@pytest.mark.parametrize("W,V,T,tp,seed", [(2, 3001, 0.8, 0.9, 1), (3, 4099, 1.0, 0.5, 2), (5, 2000, 0.7, 0.95, 3),
                                           (4, 777, 1.3, 1.0, 4)])
def test_shard_partials_rebuild_the_row(W, V, T, tp, seed):
    rng = np.random.default_rng(seed)
    z = (rng.standard_normal(V) * 3).astype(np.float32)
    z[rng.integers(0, V)] = z.max()  # a tie for the maximum: the lower index wins
    whole = O.row_stats(z, T, tp)
    shards = [vocab_shard(V, W, r) for r in range(W)]
    # 1. max / arg-max merged in rank order (value desc, index asc)
    best_v, best_i = -np.inf, -1
    for v0, vs in shards:
        j = int(np.argmax(z[v0:v0 + vs]))
        v, i = float(z[v0 + j]), v0 + j
        if best_i < 0 or v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    assert best_v == whole.max and best_i == int(np.argmax(z))
    # 2. integer mass sums
    E = _masses(z, best_v, T)
    sums = [int(E[v0:v0 + vs].sum()) for v0, vs in shards]
    assert sum(sums) == whole.sum
    # 3. top-p: digits 3..0 from summed shard histograms
    key = _key(z)
    if tp < 1.0:
        total = sum(sums)
        thr = max(1, (total * O.top_p_q32(tp)) >> 32)
        prefix, G, last = 0, 0, 0
        for d in (3, 2, 1, 0):
            hist = np.zeros(256, dtype=np.uint64)
            for v0, vs in shards:
                ks, es = key[v0:v0 + vs], E[v0:v0 + vs]
                sel = np.ones(vs, bool) if d == 3 else (ks >> np.uint64(8 * d + 8)) == (prefix >> (8 * d + 8))
                np.add.at(hist, ((ks[sel] >> np.uint64(8 * d)) & np.uint64(255)).astype(np.int64), es[sel])
            digit, G, last = _select(hist, thr, G)
            prefix |= digit << (8 * d)
        assert prefix == whole.tau and G + last == whole.nuc
        tau, nuc = prefix, G + last
    else:
        tau, nuc = 0, sum(sums)
    # 4. the draw: each shard's best (score, index) over its slice, merged
    #    (score desc, index asc); the uniforms are those of the global index
    c = O.temp_coeff(T)
    L = O.lib()
    for step in range(6):
        best, bs = -1, None
        for v0, vs in shards:
            lb, ls = -1, None
            for j in range(v0, v0 + vs):
                if key[j] < tau or E[j] == 0:
                    continue
                sc = L.orc_race_key(float(E[j]), L.orc_gumbel_uniform(seed, step, 1, 2, O.U_GUMBEL_RESAMPLE, j))
                if lb < 0 or sc > ls:
                    lb, ls = j, sc
            if lb >= 0 and (best < 0 or ls > bs or (ls == bs and lb < best)):
                best, bs = lb, ls
        assert best == O.draw_row(z, T, tp, seed, step, 1, 2, O.U_GUMBEL_RESAMPLE), step


def _tbin(t):
    """Device bin of an exponent t >= -14: floor((t + 14) * fp32(256 / 14)), at most 255."""
    b = ((t - np.float32(-14.0)).astype(np.float32) * (np.float32(256.0) / np.float32(14.0))).astype(np.float32)
    return np.minimum(b.astype(np.int64), 255)


@pytest.mark.parametrize("W,V,T,tp,scale,seed", [(2, 30001, 0.7, 0.9, 3.0, 5), (4, 20000, 0.8, 0.95, 3.0, 6),
                                                 (8, 40000, 0.7, 0.5, 4.0, 7), (3, 9999, 0.3, 0.99, 2.0, 8)])
def test_listed_shard_path_rebuilds_the_threshold(W, V, T, tp, scale, seed):
    """The listed path (specdec_shard_mass_hist / _cross / _union_select):
    per shard the mass sum, the listed mass and the t-bin histogram of the
    elements with t = (z - max) * c >= -14; summed over shards, the crossing
    bin and the mass G above it; the shards' listed elements in that bin; a
    radix select over them above G -- the oracle's tau and nucleus mass."""
    rng = np.random.default_rng(seed)
    z = (rng.standard_normal(V) * scale).astype(np.float32)
    whole = O.row_stats(z, T, tp)
    m = np.float32(whole.max)
    c = np.float32(O.temp_coeff(T))
    t = ((z - m).astype(np.float32) * c).astype(np.float32)
    E = _masses(z, m, T)
    key = _key(z)
    shards = [vocab_shard(V, W, r) for r in range(W)]
    S = 0
    ls = 0
    hist = np.zeros(256, dtype=np.uint64)
    for v0, vs in shards:
        sl = slice(v0, v0 + vs)
        S += int(E[sl].sum())
        lst = t[sl] >= np.float32(-14.0)
        ls += int(E[sl][lst].sum())
        np.add.at(hist, _tbin(t[sl][lst]), E[sl][lst])
    assert S == whole.sum
    thr = max(1, (S * O.top_p_q32(tp)) >> 32)
    assert ls >= thr  # peaked rows: the nucleus lies among the listed elements
    b, G, _ = _select(hist, thr, 0)
    cand = []
    for v0, vs in shards:
        sl = slice(v0, v0 + vs)
        sel = (t[sl] >= np.float32(-14.0)) & (_tbin(np.maximum(t[sl], np.float32(-14.0))) == b)
        cand += list(zip(key[sl][sel].tolist(), E[sl][sel].tolist()))
        assert sel.sum() <= 32
    prefix, last = 0, 0
    for d in (3, 2, 1, 0):
        h = np.zeros(256, dtype=np.uint64)
        for kk, e in cand:
            if d == 3 or (kk >> (8 * d + 8)) == (prefix >> (8 * d + 8)):
                h[(kk >> (8 * d)) & 255] += np.uint64(e)
        digit, G, last = _select(h, thr, G)
        prefix |= digit << (8 * d)
    assert prefix == whole.tau and G + last == whole.nuc
