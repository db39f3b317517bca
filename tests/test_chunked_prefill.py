"""specdec.ChunkedPrefillState against the reference's own ChunkedPrefillState
(server/chunked_prefill.cpp:4-29): the golden vectors of
tests/golden/gen_chunk_golden.py record, call by call, what the compiled
reference class returns; the mirror reproduces every call (chunk length,
first token, remaining tokens, completion), resets included.  The engine side
of chunked prefill is tested on the GPU (test_gpu_chunked_prefill.py)."""
import os

import numpy as np

import specdec as S

HERE = os.path.dirname(os.path.abspath(__file__))


def test_chunk_state_matches_reference_golden():
    g = np.load(os.path.join(HERE, "golden", "chunk_golden.npz"))
    for (n, chunk, reset_after), rec, k in zip(g["cases"].tolist(), g["records"], g["ncalls"].tolist()):
        toks = (np.arange(n, dtype=np.int32) * 7 + 3).tolist()
        st = S.ChunkedPrefillState(toks, chunk)
        for i in range(k):
            c = st.get_next_chunk()
            got = [len(c), c[0] if c else -1, st.get_remaining_tokens(), int(st.is_prefill_complete)]
            assert got == rec[i].tolist(), (n, chunk, reset_after, i)
            if i == reset_after:
                st.reset()


def test_chunks_cover_the_prompt_once():
    toks = list(range(1000, 1203))
    st = S.ChunkedPrefillState(toks, 64)
    seen, finals = [], []
    while True:
        c = st.get_next_chunk()
        if not c:
            break
        seen += c
        finals.append(st.is_prefill_complete)
    assert seen == toks and finals == [False, False, False, True]


def test_advance_offset_skips_a_shared_prefix():
    st = S.ChunkedPrefillState(list(range(100)), 64)
    st.advance_offset(48)
    assert st.get_remaining_tokens() == 52
    assert st.get_next_chunk() == list(range(48, 100)) and st.is_prefill_complete
    st2 = S.ChunkedPrefillState(list(range(10)), 4)
    st2.advance_offset(50)
    assert st2.is_prefill_complete and st2.get_next_chunk() == []
