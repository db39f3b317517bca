"""End-to-end parity of the step engine at the benchmark's model shape, and the
free-running accepted-token parity rate.

The Llama-3-8B shape (hidden 4096, 32 / 8 heads of 128, FFN 14336, vocab
128256, 3 MTP heads) is cut to 2 decoder layers so that the oracle finishes in
seconds; every kernel of the step runs at its benchmark shape per layer: the
QKV projection with RoPE and the paged K/V write in its epilogue at head dim
128, attention over 2048- and 4096-token contexts, the SwiGLU gate/up GEMM at
F = 14336, the down projection at K = 14336, the lm_head at V = 128256.

Per step: logits within 2e-2 absolute of the oracle's (draft and target),
arg-max agreement wherever the top-2 margin is >= 1e-2, drafts and acceptance
bit-exact on the engine's own logits, block tables and lengths bit-exact, the
K/V the QKV epilogue wrote for the accepted rows within the fp16 tolerance.

The free-running rate (see tests/freerun.py) is measured on the tiny
configuration (prompt of 512, chain 3, T = 1.0, seed 0) and on the cut 8B
shape (batch 4, 2048-token contexts, chain 4, T = 0.8 and greedy).
"""
import numpy as np
import pytest

import oracle as O
import specdec as S
from freerun import free_running
from helpers import margin_ok

pytestmark = pytest.mark.gpu

SHAPE8 = dict(S.MODEL_SHAPES["llama3-8b"], layers=2)
CFG8 = dict(SHAPE8, block_size=16, rms_eps=1e-5, rope_theta=10000.0)
TINY = S.MODEL_SHAPES["tiny"]
CFG_TINY = dict(TINY, block_size=16, rms_eps=1e-5, rope_theta=10000.0)
LOGIT_TOL = 2e-2
RATE_TARGET = 0.95


@pytest.fixture(scope="module")
def oracle8():
    m = O.OracleModel(CFG8, seed=1, rope_max_pos=4400)
    yield m
    m.close()


def _check_logits(got, ref, what):
    err = float(np.abs(got - ref).max())
    assert err < LOGIT_TOL, f"{what}: max |logit diff| {err}"
    rows = got.reshape(-1, got.shape[-1])
    refr = ref.reshape(-1, ref.shape[-1])
    bad = [i for i in range(rows.shape[0]) if margin_ok(refr[i]) and int(rows[i].argmax()) != int(refr[i].argmax())]
    assert not bad, f"{what}: arg-max differs where the top-2 margin >= 1e-2 (rows {bad})"
    return err


def _mirror(eng, B, ctx0):
    """Oracle KV pool (a copy of the engine's) and a block manager replaying
    the engine's appends so far (seed_state appends ctx0[b] in request order)."""
    mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
    kvo = O.OracleKV(eng.shape["layers"], nb, eng.shape["n_kv_heads"], 16, eng.shape["head_dim"])
    kvo.pool[:] = eng.read("kv", np.uint16, kvo.pool.shape)
    bm = O.BlockManager(nb, 16, B, mb)
    for b in range(B):
        bm.append(b, int(ctx0[b]))
    return kvo, bm, mb


def _tables(bm, B, mb):
    tab = np.full((B, mb), -1, np.int32)
    for b in range(B):
        t, _ = bm.table(b)
        tab[b, :len(t)] = t
    return tab


def test_8b_shape_chain_steps_match_oracle(cuda_device, oracle8):
    B, k, T, seed = 4, 4, 0.8, 1
    V, H, L = SHAPE8["vocab"], SHAPE8["hidden"], SHAPE8["layers"]
    R = k + 1
    ctx0 = np.array([2048, 2000, 1931, 2047], np.int32)
    eng = S.Engine(SHAPE8, batch=B, draft_len=k, max_ctx=2200, temperature=T, seed=seed, use_graph=True)
    eng.init_weights(1)
    eng.seed_state(ctx0, 7)
    kvo, bm, mb = _mirror(eng, B, ctx0)
    chain = np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64)
    errs = []
    for step in range(3):
        h0_prev = eng.read("h0", np.float32, (B, H))
        pend_prev = eng.read("pending", np.int32, (B,))
        lens_prev = eng.read("lens", np.int32, (B,)).copy()
        kv_prev = kvo.pool.copy()
        acc, out = eng.step_host()
        dl = eng.read("draft_logits", np.float32, (B, k, V))
        drafts = eng.read("drafts", np.int32, (B, k))
        lg = eng.read("logits", np.float32, (B, R, V))
        # decisions, bit-exact on the engine's data
        assert O.sample_rows(dl.reshape(B * k, V), k, T, 1.0, seed, step).reshape(B, k).tolist() == drafts.tolist()
        acc_o, out_o = O.accept_chain(lg, dl, drafts, T, 1.0, seed, step)
        assert acc.tolist() == acc_o.tolist() and out.tolist() == out_o.tolist()
        # numerics: the draft chain and the verify forward from the pre-step state
        dl_o, _, _ = O.draft_chain(oracle8, h0_prev, k, T, 1.0, seed, step)
        errs.append(_check_logits(dl, dl_o, f"draft logits step {step}"))
        for b in range(B):
            bm.append(b, R)
        tab = _tables(bm, B, mb)
        toks = np.concatenate([pend_prev[:, None], drafts], axis=1).reshape(-1).astype(np.int32)
        pos = np.concatenate([lens_prev[b] + np.arange(R) for b in range(B)]).astype(np.int32)
        kvo.pool[:] = kv_prev
        lg_o, hid_o = O.forward(oracle8, kvo, tab, lens_prev, toks, pos, pos, chain, B, R)
        errs.append(_check_logits(lg, lg_o.reshape(B, R, V), f"target logits step {step}"))
        # the K/V rows the QKV epilogue wrote (RoPE at head dim 128, paged slots) for the accepted rows
        kv_now = eng.read("kv", np.uint16, kvo.pool.shape)
        for b in range(B):
            for r in range(int(acc[b]) + 1):
                s = int(lens_prev[b]) + r
                blk = tab[b, s // 16]
                np.testing.assert_allclose(O.f16_vals(kv_now[:, blk, :, :, s % 16]),
                                           O.f16_vals(kvo.pool[:, blk, :, :, s % 16]), atol=2e-2, rtol=2e-2)
        # the next draft hidden state is the accepted row's final hidden state
        h0 = eng.read("h0", np.float32, (B, H))
        for b in range(B):
            ref = hid_o[b * R + int(acc[b])]
            np.testing.assert_allclose(h0[b], ref, rtol=2e-2, atol=2e-2 * float(np.abs(ref).max()))
        # commit / rollback
        for b in range(B):
            bm.truncate(b, int(lens_prev[b] + acc[b] + 1))
        np.testing.assert_array_equal(eng.read("tables", np.int32, (B, mb)), _tables(bm, B, mb))
        assert eng.read("lens", np.int32, (B,)).tolist() == (lens_prev + acc + 1).tolist()
        kvo.pool[:] = kv_now
    print(f"8b-shape chain: max |logit diff| {max(errs):.3e}")
    eng.close()


@pytest.mark.parametrize("T", [1.0, 0.0])
def test_8b_shape_tree_step_matches_oracle(cuda_device, oracle8, T):
    """One 64-node tree step (levels 1 + 4 + 16 + 32 + 11, top-4/4/2/2) over
    4096-token contexts, greedy and T = 1."""
    B, seed = 2, 2
    V, H, L = SHAPE8["vocab"], SHAPE8["hidden"], SHAPE8["layers"]
    br = [4, 4, 2, 2]
    ctx0 = np.array([4090, 4001], np.int32)
    eng = S.Engine(SHAPE8, batch=B, draft_len=0, max_ctx=4200, temperature=T, seed=seed, tree_branching=br,
                   tree_nodes=64, use_graph=True)
    eng.init_weights(1)
    eng.seed_state(ctx0, 5)
    R = eng.rows
    assert R == 64
    parent, depth, rank, anc = O.tree_build(br, 64)
    kvo, bm, mb = _mirror(eng, B, ctx0)
    h0_prev = eng.read("h0", np.float32, (B, H))
    pend_prev = eng.read("pending", np.int32, (B,))
    acc, out = eng.step_host()
    dl = eng.read("draft_logits", np.float32, (B, 4, V))
    node_tokens = eng.read("node_tokens", np.int32, (B, R))
    lg = eng.read("logits", np.float32, (B, R, V))
    path = eng.read("path", np.int32, (B, R))
    for b in range(B):
        assert node_tokens[b, 0] == pend_prev[b]
        for lv in range(4):
            topk = np.zeros(4, np.int32)
            O.lib().orc_topk(O.ptr(np.ascontiguousarray(dl[b, lv])), V, 4, O.ptr(topk))
            for n in range(1, R):
                if depth[n] == lv + 1:
                    assert node_tokens[b, n] == topk[rank[n]]
    acc_o, path_o, out_o = O.accept_tree(lg, node_tokens, parent, T, 1.0, seed, 0)
    assert acc.tolist() == acc_o.tolist() and out.tolist() == out_o.tolist() and path.tolist() == path_o.tolist()
    dl_o, _, _ = O.draft_chain(oracle8, h0_prev, 4, T, 1.0, seed, 0)
    _check_logits(dl, dl_o, "tree draft logits")
    for b in range(B):
        bm.append(b, R)
    tab = _tables(bm, B, mb)
    pos = np.concatenate([ctx0[b] + depth for b in range(B)]).astype(np.int32)
    slot = np.concatenate([ctx0[b] + np.arange(R) for b in range(B)]).astype(np.int32)
    lg_o, _ = O.forward(oracle8, kvo, tab, ctx0, node_tokens.reshape(-1), pos, slot, anc, B, R)
    _check_logits(lg, lg_o.reshape(B, R, V), "tree target logits")
    # the accepted path's K/V (written at ctx + node) now sits at ctx + 1 .. ctx + a
    kv_now = eng.read("kv", np.uint16, kvo.pool.shape)
    for b in range(B):
        for t in range(int(acc[b])):
            src, dst = int(ctx0[b] + path[b, t]), int(ctx0[b] + t + 1)
            np.testing.assert_allclose(O.f16_vals(kv_now[:, tab[b, dst // 16], :, :, dst % 16]),
                                       O.f16_vals(kvo.pool[:, tab[b, src // 16], :, :, src % 16]), atol=2e-2, rtol=2e-2)
    for b in range(B):
        bm.truncate(b, int(ctx0[b] + acc[b] + 1))
    np.testing.assert_array_equal(eng.read("tables", np.int32, (B, mb)), _tables(bm, B, mb))
    eng.close()


def test_free_running_parity_rate_tiny(cuda_device):
    """C1: tiny model, batch 1, 512-token prompt through both prefills, chain 3,
    T = 1.0, seed 0; 24 free-running steps."""
    B, k, T, seed = 1, 3, 1.0, 0
    model = O.OracleModel(CFG_TINY, seed=0, rope_max_pos=1024 + 80)
    try:
        eng = S.Engine(TINY, batch=B, draft_len=k, max_ctx=1024, temperature=T, seed=seed, use_graph=True)
        eng.init_weights(0)
        prompt = np.random.default_rng(0).integers(0, TINY["vocab"], (B, 512)).astype(np.int32)
        eng.prefill(prompt)
        mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
        kvo = O.OracleKV(TINY["layers"], nb, TINY["n_kv_heads"], 16, TINY["head_dim"])
        bm = O.BlockManager(nb, 16, B, mb)
        chain = np.array([(1 << (r + 1)) - 1 if r < 63 else (1 << 64) - 1 for r in range(64)], np.uint64)
        ctx = 0
        for c0 in range(0, 511, 64):  # the oracle's own prefill (its K/V, its final hidden state)
            Rp = min(64, 511 - c0)
            bm.append(0, Rp)
            pos = np.arange(ctx, ctx + Rp, dtype=np.int32)
            _, hidden = O.forward(model, kvo, _tables(bm, B, mb), [ctx], prompt[0, c0:c0 + Rp], pos, pos,
                                  chain[:Rp], B, Rp)
            ctx += Rp
        np.testing.assert_array_equal(eng.read("tables", np.int32, (B, mb)), _tables(bm, B, mb))
        eng.write("h0", np.ascontiguousarray(hidden[-1:], np.float32))  # both sides start from the oracle's state
        eng.write("kv", kvo.pool)
        res = free_running(eng, model, B, k, T, seed, 24, kvo, bm, mb)
        eng.close()
    finally:
        model.close()
    print(f"free-running parity (tiny, T=1.0): {res}")
    assert res["rate"] >= RATE_TARGET, res


@pytest.mark.parametrize("T", [0.8, 0.0])
def test_free_running_parity_rate_8b_shape(cuda_device, oracle8, T):
    """Cut 8B shape: batch 4, 2048-token contexts, chain 4; 8 free-running steps."""
    B, k, seed = 4, 4, 1
    ctx0 = np.array([2048, 2048, 2048, 2048], np.int32)
    eng = S.Engine(SHAPE8, batch=B, draft_len=k, max_ctx=2200, temperature=T, seed=seed, use_graph=True)
    eng.init_weights(1)
    eng.seed_state(ctx0, 11)
    kvo, bm, mb = _mirror(eng, B, ctx0)
    res = free_running(eng, oracle8, B, k, T, seed, 8, kvo, bm, mb)
    eng.close()
    print(f"free-running parity (8b shape, 2 layers, T={T}): {res}")
    assert res["rate"] >= RATE_TARGET, res
