"""The allocation-free chain acceptance entry point.

specdec_accept_chain_noalloc exists for callers that may not allocate device
memory at the moment they accept drafts (for example a serving loop that
reserved its whole device-memory budget at start-up, or a host program that
owns the GPU allocator).  It must produce exactly what specdec_accept_chain
produces with a caller-provided workspace, on consecutive calls that reuse
its fixed scratch array, and it must refuse batches larger than that array.
This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

import specdec as S
from helpers import dev, empty, ptr, stream_ptr, sync

pytestmark = pytest.mark.gpu


def _accept(lib_fn, tgt, dr, drafts, T, tp, seed, step, with_ws):
    import torch

    B, k1, V = tgt.shape
    k = k1 - 1
    d_t, d_d, d_dr = dev(tgt), dev(dr), dev(drafts)
    acc = empty(B, torch.int32)
    out = empty((B, k + 1), torch.int32)
    sp = S.sampling(T, tp, seed, step)
    if with_ws:
        ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
        ws = empty(ws_b, torch.uint8)
        S.check(lib_fn(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out), ptr(ws), ws_b,
                       stream_ptr()))
    else:
        S.check(lib_fn(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out), stream_ptr()))
    sync()
    return acc.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("T,tp,k", [(0.7, 0.9, 4), (1.0, 0.5, 3), (0.9, 1.0, 17), (0.0, 1.0, 17), (0.8, 1.0, 4),
                                    (0.0, 1.0, 4)])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda_device, T, tp, k):
    """top_p < 1, or more than 16 drafts, run the row-statistics path that
    keeps its per-row scratch in the fixed array; greedy and top_p = 1 with
    at most 16 drafts use no scratch.  The larger call comes first, so the
    second call reuses an array holding the first call's rows."""
    L = S.lib()
    for call, (B, V, seed) in enumerate([(12, 20000, 11), (5, 32000, 12)]):
        rng = np.random.default_rng(100 + call + 10 * k)
        tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
        dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
        drafts = rng.integers(0, V, (B, k)).astype(np.int32)
        drafts[:, 0] = tgt[:, 0].argmax(-1)
        drafts[:, 1] = dr[:, 1].argmax(-1)
        ref = _accept(L.specdec_accept_chain, tgt, dr, drafts, T, tp, seed, call, True)
        got = _accept(L.specdec_accept_chain_noalloc, tgt, dr, drafts, T, tp, seed, call, False)
        # integer outputs: exact agreement
        assert got[0].tolist() == ref[0].tolist(), f"call {call}: accepted lengths differ"
        assert got[1].tolist() == ref[1].tolist(), f"call {call}: emitted tokens differ"


def test_noalloc_takes_any_batch_where_it_needs_no_scratch(cuda_device):
    """Greedy acceptance of 2048 sequences x 7 drafts (16384 rows, beyond the
    fixed array) runs the sliced kernel, which needs no row scratch."""
    B, k, V = 2048, 7, 64
    rng = np.random.default_rng(3)
    tgt = rng.standard_normal((B, k + 1, V)).astype(np.float32)
    drafts = tgt[:, :k].argmax(-1).astype(np.int32)
    drafts[::3, 2] = (drafts[::3, 2] + 1) % V
    dr = np.zeros((B, k, V), np.float32)
    ref = _accept(S.lib().specdec_accept_chain, tgt, dr, drafts, 0.0, 1.0, 5, 0, True)
    got = _accept(S.lib().specdec_accept_chain_noalloc, tgt, dr, drafts, 0.0, 1.0, 5, 0, False)
    assert got[0].tolist() == ref[0].tolist() and got[1].tolist() == ref[1].tolist()


def test_noalloc_rejects_batches_beyond_its_fixed_scratch(cuda_device):
    import torch

    B, k, V = 1000, 4, 8  # 1000 * (5 + 4) rows > 8192 on the row-statistics path (top_p < 1)
    t = torch.zeros((B, k + 1, V), dtype=torch.float32, device="cuda")
    d = torch.zeros((B, k, V), dtype=torch.float32, device="cuda")
    dr = torch.zeros((B, k), dtype=torch.int32, device="cuda")
    acc = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros((B, k + 1), dtype=torch.int32, device="cuda")
    sp = S.sampling(0.8, 0.9, 0, 0)
    rc = S.lib().specdec_accept_chain_noalloc(ptr(t), ptr(d), ptr(dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                              stream_ptr())
    assert rc == S.EINVAL and "fixed scratch" in S.last_error()
