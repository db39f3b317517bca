"""CPU checks of the oracle: known-answer tests, golden vectors produced by the
reference's own C++ (tests/golden/ref_golden.npz), and algorithm properties."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")


# ---------------------------------------------------------------- Philox
def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32_10
    assert [hex(x) for x in O.philox([0, 0, 0, 0], [0, 0])] == ["0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]
    assert [hex(x) for x in O.philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2)] == [
        "0x408f276d", "0x41c83b0e", "0xa20bc7c6", "0x6d5451fd"]
    assert [hex(x) for x in O.philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0])] == [
        "0xd16cfe09", "0x94fdcceb", "0x5001e420", "0x24126ea1"]


def test_exp2_fixed_point_accuracy():
    L = O.lib()
    ts = np.concatenate([np.linspace(-30, 0, 4001), [-0.5, -1.5, -0.25, 0.0]])
    got = np.array([L.orc_exp2_fx31(float(t)) for t in ts], np.float64)
    ref = np.floor(np.exp2(ts.astype(np.float32).astype(np.float64)) * 2.0 ** 31)
    # fp32 evaluation: within a few fp32 ulp of the exact value, plus the floor
    assert (np.abs(got - ref) <= np.maximum(2.0, ref * 1e-6)).all()
    assert L.orc_exp2_fx31(0.0) == 2 ** 31
    assert L.orc_exp2_fx31(1.0) == 2 ** 31  # positive inputs clamp to 0
    assert L.orc_exp2_fx31(-41.0) == 0


def test_logit_key_is_order_preserving():
    L = O.lib()
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, 7.25, np.inf], np.float32)
    keys = [L.orc_logit_key(float(v)) for v in vals]
    assert keys == sorted(keys)


# ------------------------------------------------------------ row stats
def test_row_stats_nucleus_mass_threshold():
    rng = np.random.default_rng(3)
    z = (rng.standard_normal(5000) * 3).astype(np.float32)
    for tp in (0.5, 0.9, 0.99):
        st = O.row_stats(z, 0.7, tp)
        c = O.temp_coeff(0.7)
        L = O.lib()
        masses = np.array([L.orc_exp2_fx31(float(np.float32((np.float32(v) - np.float32(st.max)) * np.float32(c))))
                           for v in z], np.uint64)
        assert int(masses.sum()) == st.sum
        keys = np.array([L.orc_logit_key(float(v)) for v in z], np.uint64)
        inn = keys >= st.tau
        thr = max(1, (st.sum * O.top_p_q32(tp)) >> 32)
        assert int(masses[inn].sum()) == st.nuc >= thr
        # removing the smallest key in the nucleus drops the mass below the threshold
        smallest = keys[inn].min()
        assert int(masses[keys > smallest].sum()) < thr


def test_sampling_distribution_matches_softmax():
    """Draws (one per step) follow softmax(z / T)."""
    rng = np.random.default_rng(5)
    V = 12
    z = rng.standard_normal(V).astype(np.float32)
    n = 20000
    counts = np.zeros(V)
    for s in range(n):
        counts[O.draw_row(z, 1.0, 1.0, 11, s, 0, 0)] += 1
    p = np.exp(z - z.max())
    p /= p.sum()
    assert np.abs(counts / n - p).max() < 0.015


def test_gumbel_draw_is_the_argmax_of_the_scores():
    """orc_draw_row = arg-max over the nucleus of the race key
    E_j / (-log2 U_j) with the draw's own element uniforms; excluded tokens
    never win, ties go to the lower index."""
    rng = np.random.default_rng(8)
    V, T, tp = 300, 0.7, 0.9
    z = (rng.standard_normal(V) * 2).astype(np.float32)
    st = O.row_stats(z, T, tp)
    c = O.temp_coeff(T)
    L = O.lib()
    for step in range(5):
        best, bs = -1, None
        for j in range(V):
            if not L.orc_row_mass(O.ptr(z), C.byref(st), c, j) or j in (3, 17):
                continue
            e = L.orc_row_mass(O.ptr(z), C.byref(st), c, j)
            sc = L.orc_race_key(float(e), L.orc_gumbel_uniform(9, step, 2, 1, O.U_GUMBEL_DRAFT, j))
            if best < 0 or sc > bs:
                best, bs = j, sc
        assert O.draw_row(z, T, tp, 9, step, 2, 1, exclude=[3, 17]) == best


def test_det_log2_and_uniform_transform_accuracy():
    """The atanh-series log2 against float64 log2, and -log2 U across the
    whole 32-bit range (including both ends and the switch at U = 1/2)."""
    L = O.lib()
    xs = np.concatenate([np.geomspace(2.0 ** -126, 2.0 ** 127, 2000), np.linspace(0.5, 2.0, 2001)]).astype(np.float32)
    for x in xs:
        got = L.orc_det_log2(float(x))
        ref = np.log2(np.float64(x))
        assert abs(got - ref) <= 2e-7 * max(1.0, abs(ref)), (x, got, ref)
    us = [0, 1, 2, 12345, 2**31 - 1, 2**31, 2**31 + 1, 3 * 2**30, 2**32 - 2, 2**32 - 1]
    us += [int(v) for v in np.random.default_rng(1).integers(0, 2**32, 2000, dtype=np.uint64)]
    for u in us:
        got = L.orc_neg_log2_uniform(u)
        ref = -np.log2((np.float64(u) + 0.5) / 2.0 ** 32)
        assert abs(got - ref) <= 4e-7 * ref + 1e-12, (u, got, ref)  # relative: tiny values keep their precision


# --------------------------------------------------- acceptance semantics
def test_greedy_chain_is_longest_matching_prefix():
    rng = np.random.default_rng(7)
    B, k, V = 6, 4, 50
    tgt = rng.standard_normal((B, k + 1, V)).astype(np.float32)
    am = tgt.argmax(-1)
    drafts = am[:, :k].copy()
    drafts[1, 0] += 1
    drafts[2, 2] = (drafts[2, 2] + 3) % V
    drafts[3, 1] = (drafts[3, 1] + 1) % V  # later positions still match: not counted
    acc, out = O.accept_chain(tgt, None, drafts, 0.0, 1.0, 0, 0)
    assert acc.tolist() == [4, 0, 2, 1, 4, 4]
    for b in range(B):
        a = acc[b]
        assert out[b, :a].tolist() == drafts[b, :a].tolist()
        assert out[b, a] == am[b, a]
        assert (out[b, a + 1:] == -1).all()


def test_rejection_sampling_acceptance_rate():
    """Per-position acceptance probability must equal sum_j min(p_j, q_j)."""
    rng = np.random.default_rng(9)
    V, T = 16, 1.0
    zp = rng.standard_normal(V).astype(np.float32)
    zq = (zp + rng.standard_normal(V) * 0.8).astype(np.float32)
    p = np.exp(zp - zp.max()); p /= p.sum()
    q = np.exp(zq - zq.max()); q /= q.sum()
    n = 4000
    tgt = np.broadcast_to(np.stack([zp, zp]), (n, 2, V)).copy()
    dr = np.broadcast_to(zq, (n, 1, V)).copy()
    drafts = np.array([[O.draw_row(zq, T, 1.0, 1, 0, b, 0)] for b in range(n)], np.int32)
    acc, out = O.accept_chain(tgt, dr, drafts, T, 1.0, 77, 0)
    assert abs(acc.mean() - np.minimum(p, q).sum()) < 0.03
    # the emitted first token is distributed as p (speculative sampling is lossless)
    first = out[:, 0]
    hist = np.bincount(first, minlength=V) / n
    assert np.abs(hist - p).max() < 0.03


def test_tree_builder_config_shape():
    parent, depth, rank, anc = O.tree_build([4, 4, 2, 2], 64)
    assert parent.size == 64 and parent[0] == -1
    assert np.bincount(depth).tolist() == [1, 4, 16, 32, 11]
    for n in range(1, 64):
        assert depth[n] == depth[parent[n]] + 1
        assert anc[n] == (anc[parent[n]] | np.uint64(1 << n))


def test_tree_greedy_walk():
    rng = np.random.default_rng(13)
    parent, depth, rank, anc = O.tree_build([2, 2], 7)
    R, V = 7, 30
    tgt = rng.standard_normal((1, R, V)).astype(np.float32)
    am = tgt[0].argmax(-1)
    tok = np.zeros((1, R), np.int32)
    tok[0, 0] = 5
    tok[0, 1], tok[0, 2] = (am[0] + 1) % V, am[0]          # node 2 matches root's argmax
    tok[0, 5], tok[0, 6] = am[2], (am[2] + 1) % V          # node 5 (child of 2) matches
    tok[0, 3], tok[0, 4] = 1, 2
    acc, path, out = O.accept_tree(tgt, tok, parent, 0.0, 1.0, 0, 0)
    assert acc[0] == 2 and path[0, :2].tolist() == [2, 5]
    assert out[0, :3].tolist() == [am[0], am[2], am[5]]


# ----------------------------------------------- reference compatibility
def test_compat_argmax_lane_rule_known_answers():
    L = O.lib()
    z = np.zeros(16, np.float32)
    z[5] = 5.0   # lane 1
    z[12] = 5.0  # lane 0 -> the reference's 4-lane scan returns 12, not 5
    assert L.orc_compat_argmax(O.ptr(z), 16, 4, -1) == 12
    assert O.lib().orc_argmax(O.ptr(z), 16) == 5
    z2 = np.full(8, -np.inf, np.float32)
    assert L.orc_compat_argmax(O.ptr(z2), 8, 4, -1) == 0


def test_compat_verify_counts_matches_not_prefix():
    V = 8
    logits = np.zeros((1, 3, V), np.float32)
    best = [2, 3, 4]
    for i, t in enumerate(best):
        logits[0, i, t] = 1.0
    drafts = np.array([[2, 7, 4]], np.int32)  # match, mismatch, match
    acc, rep = O.compat_verify(logits, drafts, np.array([3], np.int32), V, 3)
    assert acc.tolist() == [2]
    assert rep.tolist() == [best[2]]  # replacement is best[count], lib.rs:768-777
    acc, rep = O.compat_verify(logits, np.array([[2, 3, 4]], np.int32), np.array([3], np.int32), V, 3)
    assert acc.tolist() == [3] and rep.tolist() == [-1]


# --------------------------------------------------------- golden vectors
@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_paged_attention_matches_reference_cpp(golden):
    L = O.lib()
    for ci in range(3):
        M, H, bs, _ = golden[f"pa{ci}_shape"].tolist()
        q, kp, vp = golden[f"pa{ci}_q"], golden[f"pa{ci}_k"], golden[f"pa{ci}_v"]
        off, tabs, lens = golden[f"pa{ci}_off"], golden[f"pa{ci}_tables"], golden[f"pa{ci}_lens"]
        o = np.zeros((M, H), np.float32)
        L.orc_compat_paged_attention(O.ptr(q), O.ptr(kp), O.ptr(vp), O.ptr(off), O.ptr(tabs), O.ptr(lens), O.ptr(o),
                                     M, H, bs)
        np.testing.assert_allclose(o, golden[f"pa{ci}_o"], rtol=1e-5, atol=1e-6)


def test_block_tables_match_reference_cpp(golden):
    nb, bs, _, n_req = golden["kv_cfg"].tolist()
    bm = O.BlockManager(nb, bs, n_req, 32)
    for i, (kind, a, b, c) in enumerate(golden["kv_ops"].tolist()):
        ret = 0
        if kind == 0:
            ret = bm.append(a, b)
        elif kind == 1:
            bm.free_request(a)
        elif kind == 2:
            bm.share_prefix(a, b, c)
        elif kind == 3:
            bm.free_tail_blocks(a, b)
        elif kind == 4:
            ret = int(bm.evict_tokens(a, b))
        assert ret == golden["kv_ret"][i], f"op {i}"
        for r in range(n_req):
            tab, ln = bm.table(r)
            exp = golden["kv_tables"][i][r]
            assert tab == exp[exp >= 0].tolist(), f"op {i} req {r}"
            assert ln == golden["kv_lens"][i][r], f"op {i} req {r}"
        assert abs(bm.utilization() - golden["kv_util"][i]) < 1e-6


def test_verify_and_mtp_wrappers_match_reference_cpp(golden):
    acc, rep = O.compat_verify(golden["ver_logits"], golden["ver_drafts"], golden["ver_lens"],
                               golden["ver_logits"].shape[2], golden["ver_logits"].shape[1])
    assert acc.tolist() == golden["ver_acc"].tolist()
    assert rep.tolist() == golden["ver_rep"].tolist()
    W, h = golden["mtp_w"], golden["mtp_h"]
    K, H, V = W.shape
    L = O.lib()
    lg = np.zeros((K, V), np.float32)
    L.orc_compat_mtp_predict(O.ptr(h), O.ptr(W), O.ptr(lg), H, V, K)
    out = np.zeros(K, np.int32)
    L.orc_compat_mtp_sample(O.ptr(lg), O.ptr(out), V, K, 4)
    assert out.tolist() == golden["mtp_out"].tolist()


def test_flashdecoding_split_equals_softmax():
    rng = np.random.default_rng(21)
    hd, n, chunk = 32, 100, 24
    q = rng.standard_normal(hd).astype(np.float32)
    k = rng.standard_normal((n, hd)).astype(np.float32)
    v = rng.standard_normal((n, hd)).astype(np.float32)
    L = O.lib()
    C_ = (n + chunk - 1) // chunk
    po = np.zeros((C_, hd), np.float32)
    pm = np.zeros(C_, np.float32)
    ps = np.zeros(C_, np.float32)
    for c in range(C_):
        kk = np.ascontiguousarray(k[c * chunk:(c + 1) * chunk])
        vv = np.ascontiguousarray(v[c * chunk:(c + 1) * chunk])
        o = np.zeros(hd, np.float32)
        mx = np.zeros(1, np.float32)
        sm = np.zeros(1, np.float32)
        L.orc_flashdecoding_chunk(O.ptr(q), O.ptr(kk), O.ptr(vv), kk.shape[0], hd, 0.2, O.ptr(o), O.ptr(mx), O.ptr(sm))
        po[c], pm[c], ps[c] = o, mx[0], sm[0]
    out = np.zeros(hd, np.float32)
    L.orc_flashdecoding_reduce(O.ptr(po), O.ptr(pm), O.ptr(ps), C_, hd, O.ptr(out))
    s = (k @ q) * 0.2
    w = np.exp(s - s.max())
    np.testing.assert_allclose(out, (w @ v) / w.sum(), rtol=1e-4, atol=1e-5)


# ------------------------------------------------------------ W4 / model
def test_w4_packing_round_trip_and_gemm():
    packed, scales = O.synth_w4(0, 7, 96, 384)
    deq = O.w4_dequant(packed, scales)
    # every value is (q) * scale with |q| <= 8 and the group max hits |q| = 7
    s = O.f16_vals(scales)
    q = deq / np.repeat(s, 128, axis=1)
    assert np.allclose(q, np.round(q), atol=1e-2) and np.abs(q).max() <= 8
    rng = np.random.default_rng(1)
    X = O.f16_bits(rng.standard_normal((5, 384)) * 0.5)
    Y = O.w4a16_gemm(X, packed, scales)
    np.testing.assert_allclose(Y, O.f16_vals(X) @ deq.T, rtol=1e-4, atol=1e-4)


def test_ragged_group_quantisation():
    packed, scales = O.synth_w4(0, 3, 8, 1376)
    assert scales.shape == (8, 11) and packed.shape == (8, 688)
    deq = O.w4_dequant(packed, scales)
    w = np.array([[O.lib().orc_synth_value(0, 3, r * 1376 + k) for k in range(1376)] for r in range(8)], np.float32)
    assert np.abs(deq - w).max() <= np.repeat(O.f16_vals(scales), 128, axis=1)[:, :1376].max() * 0.5 + 1e-6


def test_oracle_attention_matches_numpy():
    rng = np.random.default_rng(4)
    B, R, Hq, Hkv, hd, bs = 2, 3, 4, 2, 16, 16
    ctx = np.array([20, 5], np.int32)
    nblk = 8
    kv = O.OracleKV(1, nblk, Hkv, bs, hd)
    kv.pool[:] = O.f16_bits(rng.standard_normal(kv.pool.shape))
    tables = np.array([[3, 1, -1, -1], [6, -1, -1, -1]], np.int32)
    q = O.f16_bits(rng.standard_normal((B * R, Hq, hd)))
    mask = np.array([1, 3, 7], np.uint64)
    out = np.zeros((B * R, Hq, hd), np.uint16)
    O.lib().orc_attention(O.ptr(q), C.byref(kv.s), 0, O.ptr(tables), 4, O.ptr(ctx), O.ptr(mask), B, R, Hq, O.ptr(out))
    kvf = O.f16_vals(kv.pool)
    for b in range(B):
        L = ctx[b] + R
        K = np.stack([kvf[0, tables[b, t // bs], 0, :, t % bs] for t in range(L)], 1)  # [Hkv, L, hd]
        Vv = np.stack([kvf[0, tables[b, t // bs], 1, :, t % bs] for t in range(L)], 1)
        for r in range(R):
            vis = np.array([t < ctx[b] or (int(mask[r]) >> (t - ctx[b])) & 1 for t in range(L)], bool)
            for h in range(Hq):
                g = h // (Hq // Hkv)
                s = K[g] @ O.f16_vals(q[b * R + r, h]) / np.sqrt(hd)
                s[~vis] = -np.inf
                w = np.exp(s - s.max())
                ref = (w @ Vv[g]) / w.sum()
                np.testing.assert_allclose(O.f16_vals(out[b * R + r, h]), ref, rtol=2e-3, atol=2e-3)
