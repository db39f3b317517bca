"""Shared helpers for the GPU parity tests (torch is used only for device memory)."""
import ctypes as C

import numpy as np

import oracle as O
import specdec as S


def dev(arr, device="cuda:0"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(arr)).to(device)


def ptr(t):
    return C.c_void_p(t.data_ptr())


def stream_ptr():
    import torch

    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def empty(shape, dtype, device="cuda:0"):
    import torch

    return torch.empty(shape, dtype=dtype, device=device)


def zeros(shape, dtype, device="cuda:0"):
    import torch

    return torch.zeros(shape, dtype=dtype, device=device)


def sync():
    import torch

    torch.cuda.synchronize()


def tile_w4(packed: np.ndarray, scales: np.ndarray, N: int, K: int) -> np.ndarray:
    """numpy restatement of the tiled weight layout (8448-byte units)."""
    KG = (K + 127) // 128
    units_n = ((N + 255) // 256) * 2
    Npad, Kpad = units_n * 128, KG * 128
    u = np.full((Npad, Kpad), 8, np.uint32)
    lo = packed & 15
    hi = packed >> 4
    full = np.empty((N, K), np.uint32)
    full[:, 0::2] = lo[:, : (K + 1) // 2]
    full[:, 1::2] = hi[:, : K // 2]
    u[:N, :K] = full
    sc = np.zeros((Npad, KG), np.uint16)
    sc[:N, : scales.shape[1]] = scales
    out = np.zeros((units_n, KG, 8448), np.uint8)
    uu = u.reshape(units_n, 128, KG, 16, 8)  # [un, r, kg, kc, i]
    word = np.zeros((units_n, 128, KG, 16), np.uint32)
    for i in range(8):
        j = i >> 1
        sh = (4 * j + 16) if (i & 1) else (4 * j)
        word |= uu[..., i] << np.uint32(sh)
    words = word.transpose(0, 2, 3, 1)  # [un, kg, kc, r]
    out[:, :, :8192] = words.reshape(units_n, KG, 2048).view(np.uint8).reshape(units_n, KG, 8192)
    out[:, :, 8192:] = sc.reshape(units_n, 128, KG).transpose(0, 2, 1).copy().view(np.uint8).reshape(units_n, KG, 256)
    return out.reshape(-1)


def interleave_gu(gate, up, F: int):
    """Gate/up rows of the fused SwiGLU weight: 128-row blocks alternate
    gate rows 128t.. and up rows 128t.., zero rows (nibbles 8, scale 0) past
    F.  gate/up = (packed [F, K/2], scales [F, G]); returns (packed, scales, N)."""
    units = 2 * ((F + 127) // 128)
    N = 128 * units
    packed = np.full((N, gate[0].shape[1]), 0x88, np.uint8)
    scales = np.zeros((N, gate[1].shape[1]), gate[1].dtype)
    for t in range(units // 2):
        lo, hi = 128 * t, min(F, 128 * t + 128)
        for part, (p, s) in enumerate((gate, up)):
            r0 = 256 * t + 128 * part
            packed[r0:r0 + hi - lo] = p[lo:hi]
            scales[r0:r0 + hi - lo] = s[lo:hi]
    return packed, scales, N


def margin_ok(z: np.ndarray, thr: float = 1e-2) -> bool:
    top = np.sort(z)[-2:]
    return float(top[1] - top[0]) >= thr


LOGIT_TOL = 2e-2  # the step-engine logit tolerance (absolute)


def check_logits(got, ref, what):
    """Logits within LOGIT_TOL; arg-max equal wherever the top-2 margin >= 1e-2."""
    err = np.abs(got - ref).max()
    assert err < LOGIT_TOL, f"{what}: max |logit diff| {err}"
    rows, refr = got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1])
    assert all(int(rows[i].argmax()) == int(refr[i].argmax()) for i in range(rows.shape[0]) if margin_ok(refr[i])), what


def extend_tables(tab_pre, lens_prev, R, nb):
    """Pre-step block tables extended to the step's R new slots: the context
    blocks are the engine's; a new slot past them may take any block no
    table uses (the oracle forward writes the new rows' K/V before reading)."""
    tab = tab_pre.copy()
    free = iter(sorted(set(range(nb)) - set(tab[tab >= 0].tolist())))
    for b in range(tab.shape[0]):
        have = int((tab[b] >= 0).sum())
        for j in range(have, (int(lens_prev[b]) + R + 15) // 16):
            tab[b, j] = next(free)
    return tab


def steps_match_oracle(eng, model, mc, B, k, T, seed, steps):
    """Chain steps from the engine's current state, each checked against the
    oracle: drafts and acceptance bit-exact on the engine's logits; draft and
    target logits against the oracle's draft chain and verify forward from
    the engine's pre-step state (hidden state, pending token, KV pool)."""
    V, H = mc["vocab"], mc["hidden"]
    mb, nb = eng.info("max_blocks"), eng.info("num_blocks")
    R = k + 1
    chain = np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64)
    for _ in range(steps):
        step = int(eng.read("step", np.int32, (1,))[0])
        h0_prev = eng.read("h0", np.float32, (B, H))
        pend_prev = eng.read("pending", np.int32, (B,))
        kvo = O.OracleKV(mc["layers"], nb, mc["n_kv_heads"], 16, mc["head_dim"])
        kvo.pool[:] = eng.read("kv", np.uint16, kvo.pool.shape)
        lens_prev = eng.read("lens", np.int32, (B,)).copy()
        tab_pre = eng.read("tables", np.int32, (B, mb))
        acc, out = eng.step_host()
        dl = eng.read("draft_logits", np.float32, (B, k, V))
        drafts = eng.read("drafts", np.int32, (B, k))
        lg = eng.read("logits", np.float32, (B, R, V))
        assert O.sample_rows(dl.reshape(B * k, V), k, T, 1.0, seed, step).reshape(B, k).tolist() == drafts.tolist()
        acc_o, out_o = O.accept_chain(lg, dl, drafts, T, 1.0, seed, step)
        assert acc.tolist() == acc_o.tolist() and out.tolist() == out_o.tolist()
        dl_o, _, _ = O.draft_chain(model, h0_prev, k, T, 1.0, seed, step)
        check_logits(dl, dl_o, f"draft logits step {step}")
        toks = np.concatenate([np.concatenate([[pend_prev[b]], drafts[b]]) for b in range(B)]).astype(np.int32)
        pos = np.concatenate([lens_prev[b] + np.arange(R) for b in range(B)]).astype(np.int32)
        lg_o, _ = O.forward(model, kvo, extend_tables(tab_pre, lens_prev, R, nb), lens_prev, toks, pos, pos, chain,
                            B, R)
        check_logits(lg, lg_o.reshape(B, R, V), f"target logits step {step}")
