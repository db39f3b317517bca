"""GPU parity of the individual kernels against the CPU oracle (C-ABI calls)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import dev, empty, interleave_gu, margin_ok, ptr, stream_ptr, sync, tile_w4, zeros

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")


def _i32(shape):
    import torch

    return empty(shape, torch.int32)


# ---------------------------------------------------------------- acceptance
@pytest.mark.parametrize("B,k,V,T,tp", [(5, 4, 1000, 0.0, 1.0), (6, 4, 3000, 0.8, 1.0), (7, 8, 5000, 0.7, 0.9),
                                         (3, 3, 32000, 1.0, 1.0), (4, 8, 128256, 0.7, 0.9), (32, 4, 128256, 0.8, 1.0),
                                         (9, 2, 4099, 1.0, 1.0), (9, 2, 4099, 0.0, 1.0), (1, 16, 777, 1.3, 1.0)])
def test_accept_chain_bit_exact(cuda_device, B, k, V, T, tp):
    """Greedy and top_p = 1 take the sliced cluster kernel (cluster sizes 8, 4
    and, at B = 32, 4 CTAs per sequence; V = 4099 and 777 leave ragged,
    unaligned slices), top_p < 1 the one-CTA kernel."""
    rng = np.random.default_rng(B * 1000 + V)
    tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
    # drafts: sampled from the draft distribution by the oracle, some corrupted
    drafts = O.sample_rows(dr.reshape(B * k, V), k, max(T, 1.0), tp, 9, 0).reshape(B, k)
    if T == 0.0:
        drafts = tgt[:, :k].argmax(-1).astype(np.int32)
        drafts[0, 1] = (drafts[0, 1] + 1) % V
    acc_o, out_o = O.accept_chain(tgt, dr, drafts, T, tp, 1234, 7)
    import torch

    d_t, d_d, d_dr = dev(tgt), dev(dr), dev(drafts)
    acc, out = _i32(B), _i32((B, k + 1))
    ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
    ws = empty(ws_b, torch.uint8)
    sp = S.sampling(T, tp, 1234, 7)
    S.check(S.lib().specdec_accept_chain(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                         ptr(ws), ws_b, stream_ptr()))
    sync()
    assert acc.cpu().numpy().tolist() == acc_o.tolist()
    assert out.cpu().numpy().tolist() == out_o.tolist()


@pytest.mark.parametrize("scale,T,tp", [(0.5, 1.0, 0.9), (1.0, 1.0, 0.95), (3.0, 0.7, 0.9), (8.0, 0.7, 0.5),
                                         (3.0, 0.3, 0.999)])
def test_accept_chain_topp_both_threshold_paths(cuda_device, scale, T, tp):
    """The top-p threshold from the listed high-mass elements (peaked rows:
    scale 3, 8, low temperature) and from the whole-row radix select (flat
    rows: scale 0.5, 1, whose nucleus reaches below the listed range) --
    bit-exact with the oracle either way; one row has tied maxima."""
    B, k, V = 6, 5, 50000
    rng = np.random.default_rng(int(scale * 10) + int(tp * 1000))
    tgt = (rng.standard_normal((B, k + 1, V)) * scale).astype(np.float32)
    tgt[1, 2, 100:140] = tgt[1, 2].max()  # 40 tied maxima
    dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.3 * scale).astype(np.float32)
    drafts = O.sample_rows(dr.reshape(B * k, V), k, T, tp, 9, 0).reshape(B, k)
    acc_o, out_o = O.accept_chain(tgt, dr, drafts, T, tp, 4321, 2)
    import torch

    d_t, d_d, d_dr = dev(tgt), dev(dr), dev(drafts)
    acc, out = _i32(B), _i32((B, k + 1))
    ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
    ws = empty(ws_b, torch.uint8)
    sp = S.sampling(T, tp, 4321, 2)
    S.check(S.lib().specdec_accept_chain(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                         ptr(ws), ws_b, stream_ptr()))
    sync()
    assert acc.cpu().numpy().tolist() == acc_o.tolist()
    assert out.cpu().numpy().tolist() == out_o.tolist()
    # the sampler over the same rows (its own row statistics)
    got = _i32(B * k)
    S.check(S.lib().specdec_sample_rows(ptr(d_d), B * k, k, V, C.byref(sp), ptr(got), None, 0, stream_ptr()))
    sync()
    assert got.cpu().numpy().tolist() == O.sample_rows(dr.reshape(B * k, V), k, T, tp, 4321, 2).tolist()


def test_sample_rows_topp_nonfinite_rows(cuda_device):
    """Rows with NaN or +inf logits (a NaN exponent) take the general top-p
    path (the exponent of a NaN logit counts as 0, as in the oracle); -inf
    logits under a finite maximum stay on the listed path: draws bit-exact."""
    rng = np.random.default_rng(31)
    rows, k, V = 6, 3, 20000
    z = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    z[0, 17] = np.nan
    z[1, 5] = np.inf
    z[2, 9] = -np.inf
    z[3, [1, 2, 3]] = np.nan
    z[3, 4] = np.inf
    ref = O.sample_rows(z, k, 0.7, 0.9, 77, 1)
    out = _i32(rows)
    sp = S.sampling(0.7, 0.9, 77, 1)
    d_z = dev(z)
    S.check(S.lib().specdec_sample_rows(ptr(d_z), rows, k, V, C.byref(sp), ptr(out), None, 0, stream_ptr()))
    sync()
    assert out.cpu().numpy().tolist() == ref.tolist()


@pytest.mark.parametrize("keep", [0.9, 0.1, 0.001])
def test_topp_on_masked_vocabulary_rows(cuda_device, keep):
    """Masked vocabulary (-inf outside an allowed set, as with padded or
    constrained vocabularies): the top-p acceptance and draft draws stay
    bit-exact with the oracle, down to a handful of allowed tokens."""
    rng = np.random.default_rng(int(keep * 1000) + 3)
    B, k, V = 4, 3, 32000
    tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
    allowed = rng.random(V) < keep
    allowed[:2] = True
    tgt[:, :, ~allowed] = -np.inf
    dr[:, :, ~allowed] = -np.inf
    drafts = O.sample_rows(dr.reshape(B * k, V), k, 0.8, 0.9, 9, 0).reshape(B, k)
    out = _i32(B * k)
    sp = S.sampling(0.8, 0.9, 9, 0)
    d_t, d_d, d_dr = dev(tgt), dev(dr), dev(drafts)  # held until the kernels have run
    S.check(S.lib().specdec_sample_rows(ptr(d_d), B * k, k, V, C.byref(sp), ptr(out), None, 0, stream_ptr()))
    sync()
    assert out.cpu().numpy().reshape(B, k).tolist() == drafts.tolist()
    acc_o, out_o = O.accept_chain(tgt, dr, drafts, 0.8, 0.9, 1234, 7)
    import torch

    acc, outt = _i32(B), _i32((B, k + 1))
    ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
    ws = empty(ws_b, torch.uint8)
    sp = S.sampling(0.8, 0.9, 1234, 7)
    S.check(S.lib().specdec_accept_chain(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(outt),
                                         ptr(ws), ws_b, stream_ptr()))
    sync()
    assert acc.cpu().numpy().tolist() == acc_o.tolist()
    assert outt.cpu().numpy().tolist() == out_o.tolist()


@pytest.mark.parametrize("k", [0, 3])
def test_accept_chain_zero_residual_and_bonus_only(cuda_device, k):
    """q == p with out-of-range draft tokens: the forced rejection leaves a
    zero residual, so the token is drawn from p (the fallback draw); k = 0
    draws the bonus token only."""
    B, V = 4, 2000
    rng = np.random.default_rng(5)
    tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    dr = np.ascontiguousarray(tgt[:, :k])
    if k:
        drafts = O.sample_rows(dr.reshape(B * k, V), k, 1.0, 1.0, 9, 0).reshape(B, k)
        drafts[:, 1] = -1
        drafts[2, 0] = V + 5
    else:
        drafts = np.zeros((B, 0), np.int32)
    acc_o, out_o = O.accept_chain(tgt, dr, drafts, 1.0, 1.0, 1234, 7)
    if k:
        assert acc_o.tolist() == [1, 1, 0, 1]
    import torch

    d_t = dev(tgt)
    d_d = dev(dr) if k else dev(np.zeros(1, np.float32))
    d_dr = dev(drafts) if k else dev(np.zeros(1, np.int32))
    acc, out = _i32(B), _i32((B, k + 1))
    ws_b = S.lib().specdec_accept_workspace_bytes(B * (2 * k + 1))
    ws = empty(ws_b, torch.uint8)
    sp = S.sampling(1.0, 1.0, 1234, 7)
    S.check(S.lib().specdec_accept_chain(ptr(d_t), ptr(d_d), ptr(d_dr), B, k, V, C.byref(sp), ptr(acc), ptr(out),
                                         ptr(ws), ws_b, stream_ptr()))
    sync()
    assert acc.cpu().numpy().tolist() == acc_o.tolist()
    assert out.cpu().numpy().tolist() == out_o.tolist()


@pytest.mark.parametrize("T", [0.0, 1.0])
def test_accept_tree_bit_exact(cuda_device, T):
    rng = np.random.default_rng(17)
    parent, depth, rank, anc = O.tree_build([4, 4, 2, 2], 64)
    B, R, V = 3, 64, 2000
    tgt = (rng.standard_normal((B, R, V)) * 2).astype(np.float32)
    tok = np.zeros((B, R), np.int32)
    for b in range(B):
        tops = [np.argsort(-tgt[b, 0])[:4]]  # candidates shared per level (MTP style)
        for lv in range(1, 5):
            tops.append(np.argsort(-tgt[b, min(lv, R - 1)])[:4])
        for n in range(1, R):
            tok[b, n] = tops[depth[n] - 1][rank[n]]
    acc_o, path_o, out_o = O.accept_tree(tgt, tok, parent, T, 1.0, 55, 3)
    import torch

    acc, path, out = _i32(B), _i32((B, R)), _i32((B, R))
    sp = S.sampling(T, 1.0, 55, 3)
    d_tgt, d_tok, d_par = dev(tgt), dev(tok), dev(parent)  # keep the device buffers alive across the launch
    S.check(S.lib().specdec_accept_tree(ptr(d_tgt), ptr(d_tok), ptr(d_par), B, R, V, C.byref(sp),
                                        ptr(acc), ptr(path), ptr(out), None, 0, stream_ptr()))
    sync()
    assert acc.cpu().numpy().tolist() == acc_o.tolist()
    assert path.cpu().numpy().tolist() == path_o.tolist()
    assert out.cpu().numpy().tolist() == out_o.tolist()


@pytest.mark.parametrize("T,tp", [(0.0, 1.0), (0.8, 1.0), (0.7, 0.9)])
def test_sample_rows_bit_exact(cuda_device, T, tp):
    rng = np.random.default_rng(23)
    rows, k, V = 12, 4, 32000
    z = (rng.standard_normal((rows, V)) * 2).astype(np.float32)
    ref = O.sample_rows(z, k, T, tp, 99, 5)
    out = _i32(rows)
    sp = S.sampling(T, tp, 99, 5)
    d_z = dev(z)
    S.check(S.lib().specdec_sample_rows(ptr(d_z), rows, k, V, C.byref(sp), ptr(out), None, 0, stream_ptr()))
    sync()
    assert out.cpu().numpy().tolist() == ref.tolist()


def test_compat_verify_and_reference_symbols(cuda_device):
    g = np.load(GOLDEN)
    dec = S.SpeculativeDecoder(g["ver_logits"].shape[1])
    acc, rep = dec.verify_drafts_sve2(g["ver_logits"], g["ver_drafts"], g["ver_lens"], g["ver_logits"].shape[2],
                                      g["ver_lens"].size)
    assert acc.tolist() == g["ver_acc"].tolist() and rep.tolist() == g["ver_rep"].tolist()
    # lane tie rule: 4-lane scan picks index 12 over 5
    z = np.zeros((1, 1, 16), np.float32)
    z[0, 0, 5] = z[0, 0, 12] = 5.0
    acc, rep = S.SpeculativeDecoder(1).verify_drafts_sve2(z, np.array([[3]], np.int32), np.array([1]), 16, 1)
    assert acc.tolist() == [0] and rep.tolist() == [12]
    # MTP heads through rust_sme_mtp_predict_f32 / rust_sme_mtp_sample_f32
    heads = S.MTPHeads(*g["mtp_w"].shape)
    heads.load_weights(g["mtp_w"])
    assert heads.generate_drafts(g["mtp_h"]) == g["mtp_out"].tolist()
    W, h = g["mtp_w"], g["mtp_h"]
    K, H, V = W.shape
    ref = np.zeros((K, V), np.float32)
    O.lib().orc_compat_mtp_predict(O.ptr(h), O.ptr(W), O.ptr(ref), H, V, K)
    np.testing.assert_array_equal(heads.mtp_logits.reshape(K, V), ref)


def test_compat_paged_attention_matches_reference_golden(cuda_device):
    g = np.load(GOLDEN)
    for ci in range(3):
        M, H, bs, _ = g[f"pa{ci}_shape"].tolist()
        off, flat = g[f"pa{ci}_off"], g[f"pa{ci}_tables"]
        tabs = [flat[off[m]:off[m + 1]].tolist() for m in range(M)]
        o = np.zeros((M, H), np.float32)
        S.compute_paged_attention(g[f"pa{ci}_q"], g[f"pa{ci}_k"], g[f"pa{ci}_v"], tabs, g[f"pa{ci}_lens"], o, H, bs)
        np.testing.assert_allclose(o, g[f"pa{ci}_o"], rtol=1e-4, atol=1e-5)


def test_flashdecoding_symbols(cuda_device):
    rng = np.random.default_rng(2)
    hd, n = 64, 40
    q = rng.standard_normal(hd).astype(np.float32)
    k = rng.standard_normal((n, hd)).astype(np.float32)
    v = rng.standard_normal((n, hd)).astype(np.float32)
    L = S.lib()
    po = np.zeros((2, hd), np.float32)
    pm = np.zeros(2, np.float32)
    ps = np.zeros(2, np.float32)
    for c in range(2):
        kk = np.ascontiguousarray(k[c * 20:(c + 1) * 20])
        vv = np.ascontiguousarray(v[c * 20:(c + 1) * 20])
        L.rust_sme_flashdecoding_chunk_f32(S._p(q), S._p(kk), S._p(vv), 20, hd, 0.125, S._p(po[c]),
                                           S._p(pm[c:c + 1]), S._p(ps[c:c + 1]))
    out = np.zeros(hd, np.float32)
    L.rust_sve2_flashdecoding_reduce_f32(S._p(po), S._p(pm), S._p(ps), 2, hd, S._p(out))
    s = (k @ q) * 0.125
    w = np.exp(s - s.max())
    np.testing.assert_allclose(out, (w @ v) / w.sum(), rtol=1e-4, atol=1e-5)


# ---------------------------------------------------------------- KV manager
def test_device_block_tables_match_reference_cpp(cuda_device):
    g = np.load(GOLDEN)
    nb, bs, hid, n_req = g["kv_cfg"].tolist()
    kv = S.PagedKVCache(nb, bs, hid, max_requests=n_req, max_blocks_per_request=32)
    for i, (kind, a, b, c) in enumerate(g["kv_ops"].tolist()):
        ret = 0
        if kind == 0:
            ret = kv.append_batch([a], [b])[0]
        elif kind == 1:
            kv.free_request(a)
        elif kind == 2:
            kv.share_prefix(a, b, c)
        elif kind == 3:
            kv.free_merged_blocks(a, b)
        elif kind == 4:
            ret = int(kv.evict_least_important_blocks(a, b))
        assert ret == g["kv_ret"][i], f"op {i}"
        tabs, lens = kv.get_cache_for_batch(list(range(n_req)))
        for r in range(n_req):
            exp = g["kv_tables"][i][r]
            assert tabs[r] == exp[exp >= 0].tolist(), f"op {i} req {r}"
            assert lens[r] == g["kv_lens"][i][r]
        assert abs(kv.get_utilization() - g["kv_util"][i]) < 1e-6


def test_batch_append_and_truncate_match_oracle(cuda_device):
    rng = np.random.default_rng(8)
    nb, n_req = 200, 12
    kv = S.PagedKVCache(nb, 16, 0, max_requests=n_req, max_blocks_per_request=64)
    bm = O.BlockManager(nb, 16, n_req, 64)
    for step in range(30):
        reqs = rng.permutation(n_req)[: rng.integers(1, n_req)]
        ns = rng.integers(0, 40, reqs.size)
        kv.append_batch(reqs, ns)
        for r, n in zip(reqs, ns):
            bm.append(int(r), int(n))
        if step % 3 == 2:
            tabs, lens = kv.get_cache_for_batch(range(n_req))
            new = [int(rng.integers(0, l + 1)) if rng.random() < 0.6 else -1 for l in lens]
            kv.truncate(new)
            for r, nl in enumerate(new):
                if nl >= 0:
                    bm.truncate(r, nl)
        tabs, lens = kv.get_cache_for_batch(range(n_req))
        for r in range(n_req):
            t, ln = bm.table(r)
            assert tabs[r] == t and lens[r] == ln, (step, r)


# ---------------------------------------------------------------- W4A16 GEMM
def _gemm_case(M, N, K, seed=0):
    import torch

    packed, scales = O.synth_w4(seed, 11, N, K)
    rng = np.random.default_rng(seed + M)
    X16 = O.f16_bits(rng.standard_normal((M, K)) * 0.5)
    tiled_ref = tile_w4(packed, scales, N, K)
    nbytes = S.lib().specdec_w4_tiled_bytes(N, K)
    assert nbytes == tiled_ref.size
    d_tiled = zeros(nbytes, torch.uint8)
    d_packed, d_scales = dev(packed), dev(scales)
    S.check(S.lib().specdec_w4_tile(ptr(d_packed), ptr(d_scales), N, K, ptr(d_tiled), stream_ptr()))
    sync()
    np.testing.assert_array_equal(d_tiled.cpu().numpy(), tiled_ref)
    return packed, scales, X16, d_tiled


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (4, 768, 512), (16, 512, 1376), (32, 4096, 512), (100, 1024, 384),
                                   (160, 2816, 512), (160, 512, 1376), (300, 768, 640), (1024, 512, 256)])
def test_w4a16_gemm_matches_oracle(cuda_device, M, N, K):
    """specdec_w4a16_gemm as the planner routes it: up to 64 token rows the
    GEMV kernel, above the tcgen05 tiles."""
    import torch

    packed, scales, X16, d_tiled = _gemm_case(M, N, K)
    ref = O.w4a16_gemm(X16, packed, scales)
    ws_b = S.lib().specdec_w4a16_workspace_bytes(M, N, K)
    ws = zeros(ws_b, torch.uint8)
    Y = zeros((M, N), torch.float32)
    dX = dev(X16)
    S.check(S.lib().specdec_w4a16_gemm(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 0, ptr(ws), ws_b, stream_ptr()))
    sync()
    y = Y.cpu().numpy()
    np.testing.assert_allclose(y, ref, rtol=2e-3, atol=2e-3)
    # deterministic: same bits on a second run, and add mode doubles
    Y2 = zeros((M, N), torch.float32)
    S.check(S.lib().specdec_w4a16_gemm(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y2), N, 0, ptr(ws), ws_b, stream_ptr()))
    S.check(S.lib().specdec_w4a16_gemm(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 1, ptr(ws), ws_b, stream_ptr()))
    sync()
    np.testing.assert_array_equal(Y2.cpu().numpy(), y)
    np.testing.assert_allclose(Y.cpu().numpy(), 2 * y, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("M,N,K", [(160, 4096, 1024), (16, 1024, 2048), (100, 768, 1024), (300, 640, 512),
                                   (32, 384, 384)])
def test_w4a16_gemm_every_plan_matches_oracle(cuda_device, M, N, K):
    """Every (units per CTA, k split) path the planner may pick, on one shape:
    each within the GEMM tolerance of the oracle, and add mode exact."""
    import torch

    packed, scales, X16, d_tiled = _gemm_case(M, N, K, seed=7)
    ref = O.w4a16_gemm(X16, packed, scales)
    dX = dev(X16)
    KG = (K + 127) // 128
    for qn in (1, 2):
        for split in (1, 2, 4, 8):
            if split > KG:
                continue
            Y = zeros((M, N), torch.float32)
            S.check(S.lib().specdec_w4a16_gemm_with_plan(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 0, qn, split,
                                                         stream_ptr()))
            sync()
            y = Y.cpu().numpy()
            np.testing.assert_allclose(y, ref, rtol=2e-3, atol=2e-3, err_msg=f"qn={qn} split={split}")
            S.check(S.lib().specdec_w4a16_gemm_with_plan(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 1, qn, split,
                                                         stream_ptr()))
            sync()
            np.testing.assert_allclose(Y.cpu().numpy(), 2 * y, rtol=1e-6, atol=1e-6, err_msg=f"qn={qn} split={split}")


def test_w4a16_simt_matches_tcgen05(cuda_device):
    import torch

    M, N, K = 48, 1024, 1024
    packed, scales, X16, d_tiled = _gemm_case(M, N, K, seed=3)
    ws_b = S.lib().specdec_w4a16_workspace_bytes(M, N, K)
    ws = zeros(ws_b, torch.uint8)
    Y1, Y2 = zeros((M, N), torch.float32), zeros((M, N), torch.float32)
    dX = dev(X16)
    S.check(S.lib().specdec_w4a16_gemm(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y1), N, 0, ptr(ws), ws_b, stream_ptr()))
    S.check(S.lib().specdec_w4a16_gemm_simt(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y2), N, 0, stream_ptr()))
    sync()
    np.testing.assert_allclose(Y1.cpu().numpy(), Y2.cpu().numpy(), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("M,F,K,pad", [(160, 14336, 512, 0), (1, 256, 512, 0), (5, 1376, 512, 0), (160, 1376, 1024, 8), (33, 384, 640, 0),
                                       (300, 512, 256, 0), (7, 1001, 384, 0), (64, 1792, 4096, 0)])
def test_w4a16_gemm_swiglu_matches_unfused(cuda_device, M, F, K, pad):
    """The fused gate/up GEMM + SwiGLU epilogue equals the plain GEMM over the
    same interleaved weights followed by fp16(silu(g) * u), up to one fp16 ulp
    (the epilogue's fast exp and divide are within a few fp32 ulp); g and u
    match the oracle's contraction of the separate gate / up weights."""
    import torch

    gate, up = O.synth_w4(5, 21, F, K), O.synth_w4(5, 22, F, K)
    packed, scales, N = interleave_gu(gate, up, F)
    assert N == 128 * 2 * ((F + 127) // 128)
    d_tiled = dev(tile_w4(packed, scales, N, K))
    rng = np.random.default_rng(M + F)
    X16 = O.f16_bits(rng.standard_normal((M, K)) * 0.5)
    dX = dev(X16)
    ldh = F + pad
    h = zeros((M, ldh), torch.float16)
    S.check(S.lib().specdec_w4a16_gemm_swiglu(ptr(dX), M, K, ptr(d_tiled), F, K, ptr(h), ldh, stream_ptr()))
    # the unfused GEMM on the fused call's plan: the same k-range sums, so the same g and u
    plan = (C.c_int32 * 4)()
    S.check(S.lib().specdec_w4a16_plan(M, N, K, 2, plan))
    Y = zeros((M, N), torch.float32)
    S.check(S.lib().specdec_w4a16_gemm_with_plan(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 0, 2, plan[2],
                                                 stream_ptr()))
    sync()
    y = Y.cpu().numpy().reshape(M, N // 256, 2, 128)
    g = y[:, :, 0, :].reshape(M, -1)[:, :F]
    u = y[:, :, 1, :].reshape(M, -1)[:, :F]
    np.testing.assert_allclose(g, O.w4a16_gemm(X16, *gate), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(u, O.w4a16_gemm(X16, *up), rtol=2e-3, atol=2e-3)
    with np.errstate(over="ignore"):
        ref = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float16)
    hh = h.cpu().numpy()
    got = hh[:, :F]
    err = np.abs(got.astype(np.float32) - ref.astype(np.float32))
    assert np.all(err <= np.spacing(np.abs(ref)).astype(np.float32)), float(err.max())
    assert np.all(hh[:, F:] == 0)  # the row padding is not written


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("B,R,Hq,Hkv,hd,ctx_max,tree", [(2, 5, 8, 2, 64, 100, False), (3, 5, 32, 8, 128, 700, False),
                                                        (2, 64, 8, 2, 64, 300, True), (1, 64, 32, 8, 128, 200, True),
                                                        (4, 1, 8, 8, 128, 50, False), (2, 40, 4, 1, 64, 0, False),
                                                        (1, 4, 8, 2, 64, 511, False), (1, 5, 32, 8, 128, 2100, False)])
def test_attention_matches_oracle(cuda_device, B, R, Hq, Hkv, hd, ctx_max, tree):
    import torch

    rng = np.random.default_rng(R * 7 + hd)
    ctx = rng.integers(max(0, ctx_max // 2), ctx_max + 1, B).astype(np.int32)
    max_blocks = (ctx_max + R + 15) // 16 + 1
    nblk = B * max_blocks + 3
    perm = rng.permutation(nblk)
    tables = np.full((B, max_blocks), -1, np.int32)
    for b in range(B):
        nb = (ctx[b] + R + 15) // 16
        tables[b, :nb] = perm[b * max_blocks: b * max_blocks + nb]
    kv = O.OracleKV(1, nblk, Hkv, 16, hd)
    kv.pool[:] = O.f16_bits(rng.standard_normal(kv.pool.shape))
    q = O.f16_bits(rng.standard_normal((B * R, Hq, hd)))
    if tree:
        parent, depth, rank, anc = O.tree_build([4, 4, 2, 2], R)
        mask = anc.astype(np.uint64)
    else:
        mask = np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64)
    out_o = np.zeros((B * R, Hq, hd), np.uint16)
    O.lib().orc_attention(O.ptr(q), C.byref(kv.s), 0, O.ptr(tables), max_blocks, O.ptr(ctx), O.ptr(mask), B, R, Hq,
                          O.ptr(out_o))
    ws_b = S.lib().specdec_attention_workspace_bytes(B, R, Hq, Hkv, hd, max_blocks)
    ws = zeros(ws_b, torch.uint8)
    out = zeros((B * R, Hq, hd), torch.float16)
    d_kv = dev(kv.pool[0])
    d_q, d_tab, d_ctx, d_mask = dev(q), dev(tables), dev(ctx), dev(mask)
    S.check(S.lib().specdec_attention(ptr(d_q), ptr(d_kv), nblk, Hkv, hd, ptr(d_tab), max_blocks,
                                      ptr(d_ctx), ptr(d_mask), B, R, Hq, ptr(out), ptr(ws), ws_b, stream_ptr()))
    sync()
    got = out.cpu().numpy().astype(np.float32)
    np.testing.assert_allclose(got, O.f16_vals(out_o), rtol=1e-2, atol=1e-2)


def test_w4a16_shared_workspace_across_token_tiles(cuda_device):
    """One workspace reused by GEMMs with different token tiles (as the engine
    does): every launch must still finish every split tile."""
    import torch

    shapes = [(64, 768, 512), (4, 768, 512), (160, 768, 512), (16, 768, 512), (64, 768, 512), (300, 768, 512)]
    packed, scales, _, d_tiled = _gemm_case(8, 768, 512)
    ws_b = max(S.lib().specdec_w4a16_workspace_bytes(M, N, K) for M, N, K in shapes)
    ws = zeros(ws_b, torch.uint8)
    for M, N, K in shapes:
        X16 = O.f16_bits(np.random.default_rng(M).standard_normal((M, K)) * 0.5)
        dX = dev(X16)
        Y = zeros((M, N), torch.float32)
        S.check(S.lib().specdec_w4a16_gemm(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 0, ptr(ws), ws_b,
                                           stream_ptr()))
        sync()
        np.testing.assert_allclose(Y.cpu().numpy(), O.w4a16_gemm(X16, packed, scales), rtol=2e-3, atol=2e-3)


# ------------------------------------------------ vocabulary-sharded acceptance
@pytest.mark.parametrize("W,B,k,V,T,tp,scale", [(2, 6, 4, 3001, 0.8, 0.9, 3.0), (3, 5, 3, 4099, 1.0, 1.0, 3.0),
                                                (2, 4, 4, 2000, 0.0, 1.0, 3.0), (3, 7, 8, 32000, 0.7, 0.9, 3.0),
                                                (8, 4, 7, 40000, 0.7, 0.9, 3.0), (4, 3, 3, 5003, 1.0, 0.9, 0.5)])
def test_accept_chain_vocab_sharded_matches_oracle(cuda_device, W, B, k, V, T, tp, scale):
    """W ranks (threads sharing one GPU) each hold a contiguous vocabulary
    slice of every logits row and exchange only per-row statistics; the
    decisions equal the oracle's on the whole rows, on every rank.  Shards of
    unequal width (V not a multiple of W); greedy, T > 0 without a nucleus,
    top-p through the listed path (peaked rows, up to 8 ranks) and through
    the digit passes (flat rows, scale 0.5)."""
    import threading

    import torch

    from specdec.dist import ThreadComm, accept_chain_vocab_sharded, vocab_shard

    rng = np.random.default_rng(B * 1000 + V + W)
    tgt = (rng.standard_normal((B, k + 1, V)) * scale).astype(np.float32)
    dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5 * scale / 3).astype(np.float32)
    drafts = O.sample_rows(dr.reshape(B * k, V), k, max(T, 1.0), tp, 9, 0).reshape(B, k)
    if T == 0.0:
        drafts = tgt[:, :k].argmax(-1).astype(np.int32)
        drafts[0, 1] = (drafts[0, 1] + 1) % V
    drafts[B - 1, 0] = V + 3  # out of range: rejected, the residual is the whole target row
    acc_o, out_o = O.accept_chain(tgt, dr, drafts, T, tp, 1234, 7)
    comm = ThreadComm(W)
    results = [None] * W
    errors = []

    def rank_main(r):
        try:
            v0, vs = vocab_shard(V, W, r)
            t = dev(np.ascontiguousarray(tgt[:, :, v0:v0 + vs]))
            d = dev(np.ascontiguousarray(dr[:, :, v0:v0 + vs]))
            sp = S.sampling(T, tp, 1234, 7)
            acc, out = accept_chain_vocab_sharded(t, d, dev(drafts), k, v0, sp, comm.rank_view(r))
            torch.cuda.synchronize()
            results[r] = (acc.cpu().numpy().tolist(), out.cpu().numpy().tolist())
        except Exception as e:  # noqa: BLE001 -- reported below
            errors.append(repr(e))
            comm.barrier.abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(W)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not errors, errors
    for r in range(W):
        assert results[r] == (acc_o.tolist(), out_o.tolist()), f"rank {r}"


def test_sharded_acceptor_buffers_match_oracle(cuda_device):
    """ShardedChainAcceptor (buffers allocated once, the step counter on the
    device; issued eagerly here, as thread-ranks cannot record collectives in
    a graph): two steps over the same static inputs, each equal to the
    oracle's acceptance at that step."""
    import threading

    import torch

    from specdec.dist import ShardedChainAcceptor, ThreadComm, vocab_shard

    W, B, k, V, T, tp = 3, 5, 4, 20000, 0.7, 0.9
    rng = np.random.default_rng(77)
    tgt = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    dr = (tgt[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
    drafts = O.sample_rows(dr.reshape(B * k, V), k, T, tp, 9, 0).reshape(B, k)
    want = {st: O.accept_chain(tgt, dr, drafts, T, tp, 55, st) for st in (3, 4)}
    comm = ThreadComm(W)
    results, errors = [None] * W, []

    def rank_main(r):
        try:
            v0, vs = vocab_shard(V, W, r)
            t = dev(np.ascontiguousarray(tgt[:, :, v0:v0 + vs]))
            d = dev(np.ascontiguousarray(dr[:, :, v0:v0 + vs]))
            acc = ShardedChainAcceptor(t, d, dev(drafts), k, v0, S.sampling(T, tp, 55, 3), comm.rank_view(r),
                                       graph=False)
            got = {}
            for st in (3, 4):
                a, o = acc(st)
                torch.cuda.synchronize()
                got[st] = (a.cpu().numpy().tolist(), o.cpu().numpy().tolist())
            results[r] = got
        except Exception as e:  # noqa: BLE001 -- reported below
            errors.append(repr(e))
            comm.barrier.abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(W)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for r in range(W):
        for st in (3, 4):
            assert results[r][st][0] == want[st][0].tolist() and results[r][st][1] == want[st][1].tolist(), (r, st)
