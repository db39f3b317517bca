"""Chunk-at-a-time prefill (specdec_engine_prefill_chunk) on the tiny model.

  * Fed in the reference's 64-token chunks (ChunkedPrefillState,
    server/chunked_prefill.cpp:4-24), every slot ends bit-identical to
    specdec_engine_admit of the whole prompt: K/V rows, context length, draft
    hidden state and pending token; speculative steps afterwards agree exactly.
  * Interleaved with decode steps, as the reference scheduler interleaves
    prompt chunks with decoding requests (server/continuous_scheduler.cpp:
    133-176): one chunk of slot 2's prompt between steps while slot 2 is
    inactive leaves the decoding slots' results unchanged, and slot 2 ends in
    the state a whole-prompt admission gives it.
  * Other chunk sizes change only where the forward's row chunks start:
    the state agrees within the step-engine tolerance.
"""
import numpy as np
import pytest

import oracle as O
import specdec as S

pytestmark = pytest.mark.gpu

TINY = S.MODEL_SHAPES["tiny"]
KW = dict(batch=3, draft_len=3, max_ctx=512, temperature=1.0, seed=7, use_graph=True)


def _prompts():
    rng = np.random.default_rng(21)
    return [rng.integers(0, TINY["vocab"], n).astype(np.int32) for n in (200, 64, 130)]


def _engine():
    eng = S.Engine(TINY, **KW)
    eng.init_weights(0)
    return eng


def _kv_rows(eng, b, n):
    """K/V of the first n tokens of slot b: [n, L, 2, Hkv, hd] raw fp16 bits."""
    L, Hkv, hd = TINY["layers"], TINY["n_kv_heads"], TINY["head_dim"]
    nb, mb = eng.info("num_blocks"), eng.info("max_blocks")
    pool = eng.read("kv", np.uint16, (L, nb, 2, Hkv, 16, hd))
    tab = eng.read("tables", np.int32, (eng.batch, mb))[b]
    t = np.arange(n)
    return pool[:, tab[t // 16], :, :, t % 16, :]


def _feed(eng, b, prompt, chunk, request_id):
    st = S.ChunkedPrefillState(prompt.tolist(), chunk)
    calls = 0
    while True:
        c = st.get_next_chunk()
        if not c:
            return calls
        eng.prefill_chunk(b, c, final=st.is_prefill_complete, request_id=request_id)
        calls += 1


def _state(eng, b, n):
    H = TINY["hidden"]
    return (_kv_rows(eng, b, n), int(eng.read("lens", np.int32, (eng.batch,))[b]),
            int(eng.read("pending", np.int32, (eng.batch,))[b]), eng.read("h0", np.float32, (eng.batch, H))[b])


def test_chunked_prefill_equals_admit(cuda_device):
    prompts = _prompts()
    ref, eng = _engine(), _engine()
    try:
        for b, p in enumerate(prompts):
            ref.admit(b, 100 + b, p)
            eng.retire(b)
            assert _feed(eng, b, p, 64, 100 + b) == (len(p) + 63) // 64
        for b, p in enumerate(prompts):
            kv_r, len_r, pend_r, h_r = _state(ref, b, len(p) - 1)
            kv_e, len_e, pend_e, h_e = _state(eng, b, len(p) - 1)
            assert len_e == len_r == len(p) - 1
            assert pend_e == pend_r == int(p[-1])
            assert np.array_equal(kv_e, kv_r)
            assert np.array_equal(h_e, h_r)
        for _ in range(3):
            assert [x.tolist() for x in eng.step_host()] == [x.tolist() for x in ref.step_host()]
    finally:
        eng.close()
        ref.close()


def test_chunks_interleaved_with_decode_steps(cuda_device):
    prompts = _prompts()
    ref, eng = _engine(), _engine()
    try:
        for b in (0, 1):
            ref.admit(b, 100 + b, prompts[b])
            eng.admit(b, 100 + b, prompts[b])
        ref.admit(2, 102, prompts[2])  # whole prompt up front, kept inactive meanwhile
        eng.retire(2)
        for e in (ref, eng):
            e.set_active(np.array([1, 1, 0], np.int32))
        st = S.ChunkedPrefillState(prompts[2].tolist(), 64)
        n_steps = 0
        while not st.is_prefill_complete:
            eng.prefill_chunk(2, st.get_next_chunk(), final=st.is_prefill_complete, request_id=102)
            acc_e, tok_e = eng.step_host()
            acc_r, tok_r = ref.step_host()
            assert acc_e[:2].tolist() == acc_r[:2].tolist() and tok_e[:2].tolist() == tok_r[:2].tolist()
            n_steps += 1
        assert n_steps == 3
        n = len(prompts[2]) - 1
        kv_r, len_r, pend_r, h_r = _state(ref, 2, n)
        kv_e, len_e, pend_e, h_e = _state(eng, 2, n)
        assert (len_e, pend_e) == (len_r, pend_r) == (n, int(prompts[2][-1]))
        assert np.array_equal(kv_e, kv_r) and np.array_equal(h_e, h_r)
        for e in (ref, eng):
            e.set_active(np.array([1, 1, 1], np.int32))
        for _ in range(2):
            assert [x.tolist() for x in eng.step_host()] == [x.tolist() for x in ref.step_host()]
    finally:
        eng.close()
        ref.close()


def test_other_chunk_sizes_agree_within_tolerance(cuda_device):
    prompts = _prompts()
    ref, eng = _engine(), _engine()
    try:
        for b, p in enumerate(prompts):
            ref.admit(b, 100 + b, p)
            eng.retire(b)
            _feed(eng, b, p, 50 if b != 1 else 7, 100 + b)
        for b, p in enumerate(prompts):
            kv_r, len_r, pend_r, h_r = _state(ref, b, len(p) - 1)
            kv_e, len_e, pend_e, h_e = _state(eng, b, len(p) - 1)
            assert (len_e, pend_e) == (len_r, pend_r)
            np.testing.assert_allclose(O.f16_vals(kv_e), O.f16_vals(kv_r), rtol=2e-2, atol=2e-2)
            np.testing.assert_allclose(h_e, h_r, rtol=2e-2, atol=2e-2 * float(np.abs(h_r).max()))
    finally:
        eng.close()
        ref.close()


def test_prefill_chunk_rejects_bad_prompts(cuda_device):
    eng = _engine()
    try:
        eng.retire(0)
        with pytest.raises(S.SpecdecError) as e:
            eng.prefill_chunk(0, [5], final=True)  # no K/V token before the pending one
        assert e.value.code == S.EINVAL
        with pytest.raises(S.SpecdecError) as e:
            eng.prefill_chunk(0, np.zeros(KW["max_ctx"] + 1, np.int32), final=True)
        assert e.value.code == S.EINVAL
        with pytest.raises(S.SpecdecError):
            eng.prefill_chunk(3, [1, 2], final=True)
    finally:
        eng.close()


def test_tree_engine_chunked_prefill_keeps_the_tree_mask(cuda_device):
    """A tree engine prefills under the chain mask and puts its node mask
    back: chunk-fed slots equal admitted ones, and the tree steps after them
    agree exactly."""
    kw = dict(batch=2, draft_len=0, max_ctx=512, temperature=1.0, seed=2, tree_branching=[4, 4, 2, 2],
              tree_nodes=64, use_graph=True)
    ref, eng = S.Engine(TINY, **kw), S.Engine(TINY, **kw)
    try:
        for e in (ref, eng):
            e.init_weights(0)
        prompts = _prompts()[:2]
        mask_before = eng.read("mask", np.uint64, (64,)).copy()
        for b, p in enumerate(prompts):
            ref.admit(b, 100 + b, p)
            eng.retire(b)
            _feed(eng, b, p, 64, 100 + b)
        assert np.array_equal(eng.read("mask", np.uint64, (64,)), mask_before)
        for b, p in enumerate(prompts):
            kv_r, len_r, pend_r, h_r = _state(ref, b, len(p) - 1)
            kv_e, len_e, pend_e, h_e = _state(eng, b, len(p) - 1)
            assert (len_e, pend_e) == (len_r, pend_r) and np.array_equal(kv_e, kv_r) and np.array_equal(h_e, h_r)
        for _ in range(2):
            assert [x.tolist() for x in eng.step_host()] == [x.tolist() for x in ref.step_host()]
    finally:
        eng.close()
        ref.close()


def test_chunked_admission_with_prefix_sharing_equals_admit(cuda_device):
    """The reference scheduler's admission (continuous_scheduler.cpp:77-86):
    match the prompt in the prefix index, share the source's blocks, advance
    the chunked state past them and prefill the rest chunk by chunk; insert
    the prompt when it is complete (mark_completed, :399-409).  Against
    specdec_engine_admit with the same index: the same shared token counts,
    tables that share the same source blocks, bit-identical state and steps."""
    rng = np.random.default_rng(11)
    V = TINY["vocab"]
    p0 = rng.integers(0, V, 200).astype(np.int32)
    p1 = np.concatenate([p0[:150], rng.integers(0, V, 60)]).astype(np.int32)
    p2 = np.concatenate([p1[:180], rng.integers(0, V, 21)]).astype(np.int32)
    prompts = [p0, p1, p2]
    ref, eng = _engine(), _engine()
    c_ref, c_eng = S.RadixKVCache(), S.RadixKVCache()
    try:
        shared_ref = [ref.admit(b, 100 + b, prompts[b], c_ref) for b in range(3)]
        shared_eng = []
        for b, p in enumerate(prompts):
            sh = eng.share_prefix(b, 100 + b, p, c_eng)
            st = S.ChunkedPrefillState(p.tolist(), 64)
            st.advance_offset(sh)
            while not st.is_prefill_complete:
                eng.prefill_chunk(b, st.get_next_chunk(), final=st.is_prefill_complete, request_id=100 + b)
            c_eng.insert_prefix(100 + b, p[:-1])
            shared_eng.append(sh)
        assert shared_eng == shared_ref == [0, 144, 176]
        mb = eng.info("max_blocks")
        tab = eng.read("tables", np.int32, (eng.batch, mb))
        assert tab[1, :9].tolist() == tab[0, :9].tolist() and tab[2, :11].tolist() == tab[1, :11].tolist()
        for b, p in enumerate(prompts):
            kv_r, len_r, pend_r, h_r = _state(ref, b, len(p) - 1)
            kv_e, len_e, pend_e, h_e = _state(eng, b, len(p) - 1)
            assert (len_e, pend_e) == (len_r, pend_r) and np.array_equal(kv_e, kv_r) and np.array_equal(h_e, h_r)
        for _ in range(2):
            assert [x.tolist() for x in eng.step_host()] == [x.tolist() for x in ref.step_host()]
    finally:
        eng.close()
        ref.close()
        c_ref.close()
        c_eng.close()
