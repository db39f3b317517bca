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


@pytest.mark.parametrize("T,tp", [(0.8, 1.0), (0.7, 0.9), (0.0, 1.0)])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda_device, T, tp):
    L = S.lib()
    for call, (B, k, V, seed) in enumerate([(6, 4, 32000, 11), (9, 3, 20000, 12)]):
        rng = np.random.default_rng(100 + call)
        tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
        dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
        drafts = rng.integers(0, V, (B, k)).astype(np.int32)
        drafts[:, 0] = tgt[:, 0].argmax(-1)
        ref = _accept(L.specdec_accept_chain, tgt, dr, drafts, T, tp, seed, call, True)
        got = _accept(L.specdec_accept_chain_noalloc, tgt, dr, drafts, T, tp, seed, call, False)
        # integer outputs: exact agreement
        assert got[0].tolist() == ref[0].tolist(), f"call {call}: accepted lengths differ"
        assert got[1].tolist() == ref[1].tolist(), f"call {call}: emitted tokens differ"


def test_noalloc_rejects_batches_beyond_its_fixed_scratch(cuda_device):
    import torch

    B, k, V = 1000, 4, 8  # 1000 * (5 + 4) rows > 8192
    t = torch.zeros((B, k + 1, V), dtype=torch.float32, device="cuda")
    d = torch.zeros((B, k, V), dtype=torch.float32, device="cuda")
    dr = torch.zeros((B, k), dtype=torch.int32, device="cuda")
    acc = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros((B, k + 1), dtype=torch.int32, device="cuda")
    sp = S.sampling(0.8, 1.0, 0, 0)
    rc = S.lib().specdec_accept_chain_noalloc(ptr(t), ptr(d), ptr(dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                              stream_ptr())
    assert rc == S.EINVAL and "fixed scratch" in S.last_error()
