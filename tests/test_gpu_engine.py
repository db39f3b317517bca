"""End-to-end parity of the step engine (tiny Llama-style config) against the oracle.

Checks per step:
  * decisions bit-exact on the engine's own intermediate data: drafts are
    re-sampled by the oracle from the engine's draft logits, acceptance is
    recomputed by the oracle from the engine's target / draft logits;
  * numerics: the oracle redoes the draft chain and the verify forward from
    the engine's pre-step state (hidden state, pending token, KV pool) and the
    logits agree within 2e-2 absolute; arg-max agrees wherever the top-2
    margin is >= 1e-2;
  * block tables and lengths bit-exact against the oracle block manager.
"""
import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import interleave_gu, margin_ok, tile_w4

pytestmark = pytest.mark.gpu

TINY = S.MODEL_SHAPES["tiny"]
CFG = dict(TINY, block_size=16, rms_eps=1e-5, rope_theta=10000.0)
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def oracle_model():
    m = O.OracleModel(CFG, seed=0, rope_max_pos=1024 + 80)
    yield m
    m.close()


def test_engine_weights_bit_identical_to_oracle(cuda_device):
    eng = S.Engine(TINY, batch=1, draft_len=3, max_ctx=256, temperature=1.0, seed=0, use_graph=False)
    eng.init_weights(0)
    H, V, F, hd = TINY["hidden"], TINY["vocab"], TINY["ffn"], TINY["head_dim"]
    qd, kd = TINY["n_q_heads"] * hd, TINY["n_kv_heads"] * hd
    lm = eng.read("w_lm", np.uint8, (S.lib().specdec_w4_tiled_bytes(V, H),))
    np.testing.assert_array_equal(lm, tile_w4(*O.synth_w4(0, O.T_LM, V, H), V, H))
    parts = [O.synth_w4(0, O.layer_tensor(0, w), n, H) for w, n in ((O.T_Q, qd), (O.T_K, kd), (O.T_V, kd))]
    qkv = eng.read("w_qkv0", np.uint8, (S.lib().specdec_w4_tiled_bytes(qd + 2 * kd, H),))
    np.testing.assert_array_equal(
        qkv, tile_w4(np.vstack([p[0] for p in parts]), np.vstack([p[1] for p in parts]), qd + 2 * kd, H))
    gu_packed, gu_scales, NGU = interleave_gu(*[O.synth_w4(0, O.layer_tensor(0, w), F, H) for w in (O.T_GATE, O.T_UP)],
                                              F)
    gu = eng.read("w_gu0", np.uint8, (S.lib().specdec_w4_tiled_bytes(NGU, H),))
    np.testing.assert_array_equal(gu, tile_w4(gu_packed, gu_scales, NGU, H))
    down = eng.read("w_down0", np.uint8, (S.lib().specdec_w4_tiled_bytes(H, F),))
    np.testing.assert_array_equal(down, tile_w4(*O.synth_w4(0, O.layer_tensor(0, O.T_DOWN), H, F), H, F))
    head = eng.read("w_head0", np.uint8, (S.lib().specdec_w4_tiled_bytes(H, H),))
    np.testing.assert_array_equal(head, tile_w4(*O.synth_w4(0, O.T_MTP0, H, H), H, H))
    emb = eng.read("emb", np.uint16, (V * H,))
    ref = np.zeros(V * H, np.uint16)
    O.lib().orc_synth_f16(0, O.T_EMB, 0, V * H, O.ptr(ref))
    np.testing.assert_array_equal(emb, ref)
    eng.close()


def _tables(eng, B):
    mb = eng.info("max_blocks")
    return eng.read("tables", np.int32, (B, mb)), eng.read("lens", np.int32, (B,))


def _oracle_kv(eng):
    L, hd, Hkv = TINY["layers"], TINY["head_dim"], TINY["n_kv_heads"]
    nb = eng.info("num_blocks")
    kvo = O.OracleKV(L, nb, Hkv, 16, hd)
    kvo.pool[:] = eng.read("kv", np.uint16, kvo.pool.shape)
    return kvo


def _check_logits(got, ref, what):
    err = np.abs(got - ref).max()
    assert err < LOGIT_TOL, f"{what}: max |logit diff| {err}"
    rows = got.reshape(-1, got.shape[-1])
    refr = ref.reshape(-1, ref.shape[-1])
    agree = [int(rows[i].argmax()) == int(refr[i].argmax()) for i in range(rows.shape[0]) if margin_ok(refr[i])]
    assert all(agree), f"{what}: argmax differs where the top-2 margin >= 1e-2"


@pytest.mark.parametrize("use_graph", [False, True])
def test_tiny_chain_prefill_and_steps_match_oracle(cuda_device, oracle_model, use_graph):
    B, k, T, seed = 1, 3, 1.0, 0
    V, H = TINY["vocab"], TINY["hidden"]
    eng = S.Engine(TINY, batch=B, draft_len=k, max_ctx=1024, temperature=T, seed=seed, use_graph=use_graph)
    eng.init_weights(0)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, V, (B, 512)).astype(np.int32)
    eng.prefill(prompt)
    mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
    # ---- oracle prefill: 64-token chunks of the first 511 tokens
    kvo = O.OracleKV(TINY["layers"], nb, TINY["n_kv_heads"], 16, TINY["head_dim"])
    bm = O.BlockManager(nb, 16, B, mb)
    chain = np.array([(1 << (r + 1)) - 1 if r < 63 else (1 << 64) - 1 for r in range(64)], np.uint64)
    ctx, hidden = 0, None
    for c0 in range(0, 511, 64):
        Rp = min(64, 511 - c0)
        bm.append(0, Rp)
        tab = np.full((B, mb), -1, np.int32)
        t, _ = bm.table(0)
        tab[0, :len(t)] = t
        pos = np.arange(ctx, ctx + Rp, dtype=np.int32)
        _, hidden = O.forward(oracle_model, kvo, tab, [ctx], prompt[0, c0:c0 + Rp], pos, pos, chain[:Rp], B, Rp,
                              want_logits=False)
        ctx += Rp
    h0 = eng.read("h0", np.float32, (B, H))
    np.testing.assert_allclose(h0[0], hidden[-1], rtol=2e-2, atol=2e-2 * np.abs(hidden[-1]).max())
    assert eng.read("pending", np.int32, (B,)).tolist() == [int(prompt[0, -1])]
    tables, lens = _tables(eng, B)
    t, ln = bm.table(0)
    assert tables[0, :len(t)].tolist() == t and lens[0] == ln
    # ---- speculative steps
    R = k + 1
    for step in range(4):
        h0_prev = eng.read("h0", np.float32, (B, H))
        pend_prev = eng.read("pending", np.int32, (B,))
        kv_prev = _oracle_kv(eng)
        ctx_prev = int(eng.read("lens", np.int32, (B,))[0])
        acc, out = eng.step_host()
        dl = eng.read("draft_logits", np.float32, (B, k, V))
        drafts = eng.read("drafts", np.int32, (B, k))
        lg = eng.read("logits", np.float32, (B, R, V))
        # decisions, bit-exact on the engine's data
        assert O.sample_rows(dl.reshape(B * k, V), k, T, 1.0, seed, step).reshape(B, k).tolist() == drafts.tolist()
        acc_o, out_o = O.accept_chain(lg, dl, drafts, T, 1.0, seed, step)
        assert acc.tolist() == acc_o.tolist() and out.tolist() == out_o.tolist()
        # numerics of the draft chain and of the verify forward
        dl_o, _, _ = O.draft_chain(oracle_model, h0_prev, k, T, 1.0, seed, step)
        _check_logits(dl, dl_o, f"draft logits step {step}")
        bm.append(0, R)
        tab = np.full((B, mb), -1, np.int32)
        t, _ = bm.table(0)
        tab[0, :len(t)] = t
        toks = np.concatenate([pend_prev, drafts[0]]).astype(np.int32)
        pos = np.arange(ctx_prev, ctx_prev + R, dtype=np.int32)
        lg_o, _ = O.forward(oracle_model, kv_prev, tab, [ctx_prev], toks, pos, pos, chain[:R], B, R)
        _check_logits(lg, lg_o.reshape(B, R, V), f"target logits step {step}")
        # commit / rollback of the block table
        bm.truncate(0, ctx_prev + int(acc[0]) + 1)
        tables, lens = _tables(eng, B)
        t, ln = bm.table(0)
        assert tables[0, :len(t)].tolist() == t and (tables[0, len(t):] == -1).all() and lens[0] == ln
        assert eng.read("pending", np.int32, (B,))[0] == out[0, acc[0]]
    assert eng.read("step", np.int32, (1,))[0] == 4
    eng.close()


def test_tiny_tree_step_matches_oracle(cuda_device, oracle_model):
    B, T, seed = 2, 1.0, 2
    V, H, L = TINY["vocab"], TINY["hidden"], TINY["layers"]
    br = [4, 4, 2, 2]
    eng = S.Engine(TINY, batch=B, draft_len=0, max_ctx=512, temperature=T, seed=seed, tree_branching=br,
                   tree_nodes=64, use_graph=True)
    eng.init_weights(0)
    ctx0 = np.array([120, 77], np.int32)
    eng.seed_state(ctx0, 5)
    R = eng.rows
    assert R == 64
    parent, depth, rank, anc = O.tree_build(br, 64)
    mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
    bm = O.BlockManager(nb, 16, B, mb)  # mirrors every append / rollback of the engine
    for b in range(B):
        bm.append(b, int(ctx0[b]))

    def oracle_tables():
        tab = np.full((B, mb), -1, np.int32)
        for b in range(B):
            t, _ = bm.table(b)
            tab[b, :len(t)] = t
        return tab

    for step in range(2):
        h0_prev = eng.read("h0", np.float32, (B, H))
        kv_prev = _oracle_kv(eng)
        lens_prev = eng.read("lens", np.int32, (B,)).copy()
        pend_prev = eng.read("pending", np.int32, (B,))
        acc, out = eng.step_host()
        dl = eng.read("draft_logits", np.float32, (B, 4, V))
        node_tokens = eng.read("node_tokens", np.int32, (B, R))
        lg = eng.read("logits", np.float32, (B, R, V))
        path = eng.read("path", np.int32, (B, R))
        # node tokens = top-b of the level's draft distribution, by child rank
        for b in range(B):
            assert node_tokens[b, 0] == pend_prev[b]
            for lv in range(4):
                topk = np.zeros(4, np.int32)
                z = np.ascontiguousarray(dl[b, lv])
                O.lib().orc_topk(O.ptr(z), V, 4, O.ptr(topk))
                for n in range(1, R):
                    if depth[n] == lv + 1:
                        assert node_tokens[b, n] == topk[rank[n]]
        acc_o, path_o, out_o = O.accept_tree(lg, node_tokens, parent, T, 1.0, seed, step)
        assert acc.tolist() == acc_o.tolist() and out.tolist() == out_o.tolist()
        assert path.tolist() == path_o.tolist()
        # numerics: draft chain and verify forward with the ancestor mask
        dl_o, _, _ = O.draft_chain(oracle_model, h0_prev, 4, T, 1.0, seed, step)
        _check_logits(dl, dl_o, "tree draft logits")
        for b in range(B):
            bm.append(b, R)
        tab = oracle_tables()
        pos = np.concatenate([lens_prev[b] + depth for b in range(B)]).astype(np.int32)
        slot = np.concatenate([lens_prev[b] + np.arange(R) for b in range(B)]).astype(np.int32)
        lg_o, _ = O.forward(oracle_model, kv_prev, tab, lens_prev, node_tokens.reshape(-1), pos, slot, anc, B, R)
        _check_logits(lg, lg_o.reshape(B, R, V), "tree target logits")
        # compaction: the accepted path's K/V (oracle wrote it at slot ctx+node) sits at ctx+1..ctx+a
        kv_now = eng.read("kv", np.uint16, kv_prev.pool.shape)
        for b in range(B):
            for t in range(int(acc[b])):
                src = lens_prev[b] + path[b, t]
                dst = lens_prev[b] + t + 1
                for l in range(L):
                    got = kv_now[l, tab[b, dst // 16], :, :, dst % 16]
                    want = kv_prev.pool[l, tab[b, src // 16], :, :, src % 16]
                    np.testing.assert_allclose(O.f16_vals(got), O.f16_vals(want), atol=2e-2, rtol=2e-2)
        for b in range(B):
            bm.truncate(b, int(lens_prev[b] + acc[b] + 1))
        tables, lens = _tables(eng, B)
        np.testing.assert_array_equal(tables, oracle_tables())
        assert (lens == lens_prev + acc + 1).all()
    eng.close()


def test_engine_kv_pool_starts_zeroed(cuda_device):
    """The verify attention reads whole 16-slot blocks and gives the slots past
    a sequence's length zero probability; that only holds if those slots hold
    finite values, so the pool starts as zeros (never stale device memory)."""
    import torch

    junk = torch.full((64 << 20,), float("nan"), device="cuda")  # leave NaN bits behind in freed memory
    del junk
    torch.cuda.empty_cache()
    eng = S.Engine(TINY, batch=2, draft_len=3, max_ctx=256, use_graph=False)
    L, hd, Hkv = TINY["layers"], TINY["head_dim"], TINY["n_kv_heads"]
    pool = eng.read("kv", np.uint16, (L, eng.info("num_blocks"), 2, Hkv, 16, hd))
    assert not pool.any()
    eng.close()
