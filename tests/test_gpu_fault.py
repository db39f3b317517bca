"""Failure paths on the GPU, without a fault: a bounded device-side wait that
runs out is reported as SPECDEC_ETIMEOUT through the device status word, the
word is cleared, and the context keeps computing correct results afterwards.

The wait is the same bounded mbarrier wait (about 2 s of wall time) that the
TMA / tensor-core kernels use for their producer stages; here nothing ever
completes the barrier's phase, so the wait gives up and takes the kernels'
give-up path (record the site, return)."""
import ctypes as C
import time

import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import dev, empty, ptr, stream_ptr, sync

pytestmark = pytest.mark.gpu


def _accept_greedy_matches_oracle():
    import torch

    B, k, V = 4, 3, 3000
    rng = np.random.default_rng(5)
    tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    drafts = tgt[:, :k].argmax(-1).astype(np.int32)
    drafts[1, 0] = (drafts[1, 0] + 1) % V
    acc_o, out_o = O.accept_chain(tgt, tgt[:, :k].copy(), drafts, 0.0, 1.0, 0, 0)
    acc, out = empty(B, torch.int32), empty((B, k + 1), torch.int32)
    ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
    ws = empty(ws_b, torch.uint8)
    d_t, d_dr = dev(tgt), dev(drafts)  # held until the kernels have run
    sp = S.sampling(0.0, 1.0, 0, 0)
    S.check(S.lib().specdec_accept_chain(ptr(d_t), ptr(d_t), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                         ptr(ws), ws_b, stream_ptr()))
    sync()
    return acc.cpu().numpy().tolist() == acc_o.tolist() and out.cpu().numpy().tolist() == out_o.tolist()


def test_device_wait_gives_up_with_etimeout(cuda_device):
    L = S.lib()
    assert _accept_greedy_matches_oracle()
    t0 = time.monotonic()
    rc = L.specdec_selftest_wait_timeout(stream_ptr())
    waited = time.monotonic() - t0
    assert rc == S.ETIMEOUT
    assert "site 90" in S.last_error()
    assert 1.5 < waited < 60.0  # the ~2 s limit of the wait, not a hang
    # the status word was cleared (an engine's status query reads it) and the
    # context still computes
    eng = S.Engine(S.MODEL_SHAPES["tiny"], batch=1, draft_len=3, max_ctx=128, temperature=0.0, seed=0,
                   use_graph=False)
    try:
        assert eng.info("status") == 0
    finally:
        eng.close()
    assert _accept_greedy_matches_oracle()
    # and the failure path can be taken again
    assert L.specdec_selftest_wait_timeout(stream_ptr()) == S.ETIMEOUT
    assert _accept_greedy_matches_oracle()
