"""Free-running accepted-token parity: the engine and the oracle each run their
own speculative-decoding trajectory (chain drafts) from the same starting
state, and the emitted tokens are compared step by step.

Each side drafts from its own hidden state, verifies against its own paged KV
and accepts on its own logits.  A sequence whose step emits the same accepted
length and tokens on both sides counts those tokens as matched and both sides
carry on independently.  A step that differs counts the engine's emitted
tokens as mismatched -- or as excluded, under greedy decoding, where one of the
oracle's logit rows of that step has a top-2 margin below 1e-2 (the parity rule
for arg-max decisions) -- and the oracle's state for that sequence (hidden
state, pending token, length, the sequence's K/V blocks) is set to the
engine's, so the next step compares like with like again.

rate = matched / (matched + mismatched); the target is >= 0.95.

Block tables: the oracle's block manager replays the engine's appends and
rollbacks (the lengths agree after every step, matched or resynchronised), so
both sides address the same slots and their tables are checked bit for bit.
"""
from __future__ import annotations

import numpy as np

import oracle as O


def _min_margin(rows: np.ndarray) -> float:
    r = rows.reshape(-1, rows.shape[-1])
    top = np.sort(r, axis=1)[:, -2:]
    return float(np.min(top[:, 1] - top[:, 0]))


def free_running(eng, model, B, k, T, seed, steps, oracle_kv, bm, max_blocks):
    """Runs `steps` steps on both sides from the engine's current state (the
    oracle's KV pool `oracle_kv` and block manager `bm` must mirror it).
    Returns dict(matched, mismatched, excluded, rate, steps)."""
    V, H = model.cfg["vocab"], model.cfg["hidden"]
    R = k + 1
    chain = np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64)
    h0 = eng.read("h0", np.float32, (B, H)).copy()
    pend = eng.read("pending", np.int32, (B,)).copy()
    lens = eng.read("lens", np.int32, (B,)).copy()
    step0 = int(eng.read("step", np.int32, (1,))[0])
    matched = mismatched = excluded = 0
    for i in range(steps):
        st = step0 + i
        # ---- oracle step on its own state
        dl, dr, _ = O.draft_chain(model, h0, k, T, 1.0, seed, st)
        for b in range(B):
            bm.append(b, R)
        tab = np.full((B, max_blocks), -1, np.int32)
        for b in range(B):
            t, _ = bm.table(b)
            tab[b, :len(t)] = t
        toks = np.concatenate([pend[:, None], dr], axis=1).reshape(-1).astype(np.int32)
        pos = np.concatenate([lens[b] + np.arange(R) for b in range(B)]).astype(np.int32)
        lg, hid = O.forward(model, oracle_kv, tab, lens, toks, pos, pos, chain, B, R)
        lg = lg.reshape(B, R, V)
        acc_o, out_o = O.accept_chain(lg, dl, dr, T, 1.0, seed, st)
        # ---- engine step
        acc, out = eng.step_host()
        e_lens = eng.read("lens", np.int32, (B,))
        for b in range(B):
            bm.truncate(b, int(e_lens[b]))
        e_tab = eng.read("tables", np.int32, (B, max_blocks))
        tab = np.full((B, max_blocks), -1, np.int32)
        for b in range(B):
            t, ln = bm.table(b)
            tab[b, :len(t)] = t
            assert ln == e_lens[b]
        np.testing.assert_array_equal(e_tab, tab, err_msg=f"block tables after step {st}")
        resync = []
        for b in range(B):
            a = int(acc[b])
            same = int(acc_o[b]) == a and out_o[b, :a + 1].tolist() == out[b, :a + 1].tolist()
            if same:
                matched += a + 1
                h0[b] = hid[b * R + a]
                pend[b] = out_o[b, a]
                lens[b] += a + 1
                assert lens[b] == e_lens[b]
                continue
            if T <= 0.0 and min(_min_margin(lg[b]), _min_margin(dl[b])) < 1e-2:
                excluded += a + 1
            else:
                mismatched += a + 1
            resync.append(b)
        if resync:
            e_h0 = eng.read("h0", np.float32, (B, H))
            e_pend = eng.read("pending", np.int32, (B,))
            pool = eng.read("kv", np.uint16, oracle_kv.pool.shape)
            for b in resync:
                h0[b], pend[b], lens[b] = e_h0[b], e_pend[b], e_lens[b]
                t, _ = bm.table(b)
                blocks = np.asarray(t, np.int64)
                oracle_kv.pool[:, blocks] = pool[:, blocks]
    total = matched + mismatched
    return dict(matched=matched, mismatched=mismatched, excluded=excluded, steps=steps,
                rate=(matched / total) if total else 1.0)
