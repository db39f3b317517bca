"""GPU parity at the shapes the benchmark times (Llama-3-8B and 14B shapes).

The W4A16 GEMMs of the 8B verify step (M = 160 rows: batch 32 x 5) and of
the draft (M = 32 draft-head rows, M = 128 draft lm_head rows) run on the
full-size weight matrices through the C ABI; the oracle contracts a sample of
the output columns (every column would take minutes on the host), spread over
the whole range and including the first and last 128-row tiles.  Attention at
the 14B head grouping (40 query heads over 8 KV heads) and a 64-node draft tree
over 4096-token contexts is checked against the oracle in full.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import dev, interleave_gu, ptr, stream_ptr, sync, zeros

pytestmark = pytest.mark.gpu
TOL = 2e-3  # the GEMM tolerance of the smaller-shape tests


def _weights(seed, tid, N, K):
    """Full-size synthetic int4 weights (oracle generator), tiled on the device."""
    import torch

    packed, scales = O.synth_w4(seed, tid, N, K)
    tiled = zeros(S.lib().specdec_w4_tiled_bytes(N, K), torch.uint8)
    d_p, d_s = dev(packed), dev(scales)
    S.check(S.lib().specdec_w4_tile(ptr(d_p), ptr(d_s), N, K, ptr(tiled), stream_ptr()))
    sync()
    return packed, scales, tiled


def _sample_cols(N, n=640, seed=0):
    rng = np.random.default_rng(seed)
    edge = np.concatenate([np.arange(0, 64), np.arange(N - 64, N), np.arange(N // 2 - 32, N // 2 + 32)])
    return np.unique(np.concatenate([edge, rng.choice(N, size=n, replace=False)]))


@pytest.mark.parametrize("what,M,N,K,mode", [
    ("lm_head (verify, 1002 one-unit tiles)", 160, 128256, 4096, 0),
    ("o_proj (residual add)", 160, 4096, 4096, 1),
    ("down_proj (k split, residual add)", 160, 4096, 14336, 1),
    ("qkv_proj (unfused form)", 160, 6144, 4096, 0),
    ("draft lm_head", 128, 128256, 4096, 0),
    ("draft head", 32, 4096, 4096, 0),
    ("batch-1 verify rows", 5, 4096, 14336, 1),
    ("14b lm_head", 320, 152064, 5120, 0),
])
def test_w4a16_gemm_8b_shapes_match_oracle(cuda_device, what, M, N, K, mode):
    packed, scales, tiled = _weights(1, 0x2000 + N % 997 + K, N, K)
    rng = np.random.default_rng(M + N + K)
    X16 = O.f16_bits(rng.standard_normal((M, K)))
    Y0 = (rng.standard_normal((M, N)) * 2).astype(np.float32) if mode else np.zeros((M, N), np.float32)
    Y, d_x = dev(Y0), dev(X16)
    S.check(S.lib().specdec_w4a16_gemm(ptr(d_x), M, K, ptr(tiled), N, K, ptr(Y), N, mode, None, 0, stream_ptr()))
    sync()
    cols = _sample_cols(N)
    ref = O.w4a16_gemm(X16, np.ascontiguousarray(packed[cols]), np.ascontiguousarray(scales[cols]))
    if mode:
        ref = ref + Y0[:, cols]
    got = Y.cpu().numpy()[:, cols]
    np.testing.assert_allclose(got, ref, rtol=TOL, atol=TOL, err_msg=what)


def test_w4a16_gemm_swiglu_8b_shape_matches_oracle(cuda_device):
    """gate/up + SwiGLU epilogue at F = 14336 (112 two-unit tiles): h against
    fp16(silu(g) * u) of the oracle's g and u on sampled features, within the
    GEMM tolerance carried through silu(g) * u."""
    import torch

    M, F, K = 160, 14336, 4096
    cols = _sample_cols(F, n=384, seed=1)
    gate, up = O.synth_w4(1, 0x3004, F, K), O.synth_w4(1, 0x3005, F, K)
    packed, scales, N = interleave_gu(gate, up, F)
    tiled = zeros(S.lib().specdec_w4_tiled_bytes(N, K), torch.uint8)
    d_p, d_s = dev(packed), dev(scales)
    S.check(S.lib().specdec_w4_tile(ptr(d_p), ptr(d_s), N, K, ptr(tiled), stream_ptr()))
    X16 = O.f16_bits(np.random.default_rng(9).standard_normal((M, K)))
    h, d_x = zeros((M, F), torch.float16), dev(X16)
    S.check(S.lib().specdec_w4a16_gemm_swiglu(ptr(d_x), M, K, ptr(tiled), F, K, ptr(h), F, stream_ptr()))
    sync()
    g = O.w4a16_gemm(X16, np.ascontiguousarray(gate[0][cols]), np.ascontiguousarray(gate[1][cols]))
    u = O.w4a16_gemm(X16, np.ascontiguousarray(up[0][cols]), np.ascontiguousarray(up[1][cols]))
    silu = g / (np.float32(1) + np.exp(-g))
    ref = (silu * u).astype(np.float16).astype(np.float32)
    # |d(silu(g) u)| <= (|silu'(g)| |u| + |silu(g)|) * TOL (|silu'| <= 1.1), plus one fp16 rounding
    bound = (1.1 * np.abs(u) + np.abs(silu) + 1.0) * TOL + np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    got = h.cpu().numpy().astype(np.float32)[:, cols]
    err = np.abs(got - ref)
    assert np.all(err <= bound), float((err - bound).max())


@pytest.mark.parametrize("B,R,Hq,Hkv,hd,ctx_lo,ctx_hi,tree", [
    (3, 5, 40, 8, 128, 1024, 2100, False),   # 14B grouping: 5 query heads per KV head, ragged contexts
    (2, 64, 32, 8, 128, 4090, 4096, True),   # 8B 64-node draft tree over 4096-token contexts
    (2, 64, 40, 8, 128, 3000, 4096, True),   # 14B grouping with the tree
    (4, 5, 32, 8, 128, 2048, 2048, False),   # 8B chain verify at the benchmark's context
])
def test_attention_benchmark_shapes_match_oracle(cuda_device, B, R, Hq, Hkv, hd, ctx_lo, ctx_hi, tree):
    import torch

    rng = np.random.default_rng(B * 31 + R + Hq + ctx_hi)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, B).astype(np.int32)
    max_blocks = (ctx_hi + R + 15) // 16 + 1
    nblk = B * max_blocks + 5
    perm = rng.permutation(nblk)
    tables = np.full((B, max_blocks), -1, np.int32)
    for b in range(B):
        nb = (ctx[b] + R + 15) // 16
        tables[b, :nb] = perm[b * max_blocks: b * max_blocks + nb]
    kv = O.OracleKV(1, nblk, Hkv, 16, hd)
    kv.pool[:] = O.f16_bits(rng.standard_normal(kv.pool.shape))
    q = O.f16_bits(rng.standard_normal((B * R, Hq, hd)))
    if tree:
        _, _, _, anc = O.tree_build([4, 4, 2, 2], R)
        mask = anc.astype(np.uint64)
    else:
        mask = np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64)
    out_o = np.zeros((B * R, Hq, hd), np.uint16)
    O.lib().orc_attention(O.ptr(q), C.byref(kv.s), 0, O.ptr(tables), max_blocks, O.ptr(ctx), O.ptr(mask), B, R, Hq,
                          O.ptr(out_o))
    ws_b = S.lib().specdec_attention_workspace_bytes(B, R, Hq, Hkv, hd, max_blocks)
    ws = zeros(max(ws_b, 1), torch.uint8)
    out = zeros((B * R, Hq, hd), torch.float16)
    d_q, d_kv, d_t, d_c, d_m = dev(q), dev(kv.pool[0]), dev(tables), dev(ctx), dev(mask)
    S.check(S.lib().specdec_attention(ptr(d_q), ptr(d_kv), nblk, Hkv, hd, ptr(d_t), max_blocks, ptr(d_c), ptr(d_m),
                                      B, R, Hq, ptr(out), ptr(ws), ws_b, stream_ptr()))
    sync()
    np.testing.assert_allclose(out.cpu().numpy().astype(np.float32), O.f16_vals(out_o), rtol=1e-2, atol=1e-2)
