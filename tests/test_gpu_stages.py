"""The step's four stages as separate calls (specdec_engine_draft,
_verify_forward, _accept, _kv_commit_rollback), the device-resident ABI's
draft / verify / accept / commit-rollback split.

  * Called in order they reproduce specdec_engine_step (CUDA-graph replay)
    exactly, for chain and tree engines: accepted lengths, emitted tokens and
    the sequences' state after several steps.
  * Between draft and verify a caller may replace the drafts (the reference's
    n-gram drafter, SpeculativeDecoder::generate_draft, feeds drafts this
    way): greedy acceptance then counts the drafts that equal the arg-max of
    the verify logits read back between verify and accept.
"""
import numpy as np
import pytest

import specdec as S

pytestmark = pytest.mark.gpu

TINY = S.MODEL_SHAPES["tiny"]


def _pair(**kw):
    engines = [S.Engine(TINY, **kw) for _ in range(2)]
    for e in engines:
        e.init_weights(0)
        e.seed_state(np.array([150, 70, 33][:kw["batch"]], np.int32), 4)
    return engines


def _staged(e):
    e.draft()
    e.verify_forward()
    e.accept()
    e.kv_commit_rollback()
    return (e.read("accepted", np.int32, (e.batch,)).tolist(),
            e.read("out_tokens", np.int32, (e.batch, e.rows)).tolist())


@pytest.mark.parametrize("tree", [False, True])
def test_stages_equal_the_graphed_step(cuda_device, tree):
    kw = dict(batch=3, max_ctx=512, temperature=1.0, seed=3, use_graph=True)
    kw.update(dict(draft_len=0, tree_branching=[4, 4, 2, 2], tree_nodes=64) if tree else dict(draft_len=3))
    ref, eng = _pair(**kw)
    try:
        for _ in range(4):
            acc, out = ref.step_host()
            assert _staged(eng) == (acc.tolist(), out.tolist())
        for what, dt, shape in (("lens", np.int32, (3,)), ("pending", np.int32, (3,)), ("step", np.int32, (1,))):
            assert np.array_equal(eng.read(what, dt, shape), ref.read(what, dt, shape))
        H = TINY["hidden"]
        assert np.array_equal(eng.read("h0", np.float32, (3, H)), ref.read("h0", np.float32, (3, H)))
    finally:
        ref.close()
        eng.close()


def test_replaced_drafts_are_verified_greedily(cuda_device):
    B, k, V = 3, 3, TINY["vocab"]
    eng = S.Engine(TINY, batch=B, draft_len=k, max_ctx=512, temperature=0.0, seed=5, use_graph=False)
    try:
        eng.init_weights(0)
        eng.seed_state(np.array([150, 70, 33], np.int32), 4)
        for step in range(3):
            eng.draft()
            own = eng.read("drafts", np.int32, (B, k))
            # an outside drafter's guesses: the engine's own drafts for sequence 0,
            # shifted tokens elsewhere (sequence 2 keeps its first draft)
            mine = own.copy()
            mine[1] = (own[1] + 1) % V
            mine[2, 1:] = (own[2, 1:] + 7) % V
            eng.write("drafts", mine)
            eng.verify_forward()
            logits = eng.read("logits", np.float32, (B, k + 1, V))
            eng.accept()
            acc = eng.read("accepted", np.int32, (B,))
            out = eng.read("out_tokens", np.int32, (B, k + 1))
            best = logits.argmax(-1)
            for b in range(B):
                a = 0
                while a < k and mine[b, a] == best[b, a]:
                    a += 1
                assert acc[b] == a, (step, b)
                assert out[b, :a + 1].tolist() == best[b, :a + 1].tolist()
            eng.kv_commit_rollback()
    finally:
        eng.close()
