"""Generates tests/golden/ref_golden.npz by running the reference's own C++
(compiled by oracle/build_ref.sh into oracle/_ref/libref.so) on seeded inputs.

Pinned by these vectors:
  * compute_paged_attention (server/paged_attention.cpp:16-111), run unmodified;
  * PagedKVCache block tables / lengths / utilisation after a scripted sequence
    of append, free, share_prefix, free_merged_blocks and evict calls
    (server/paged_kv_cache.cpp:50-228), run unmodified;
  * SpeculativeDecoder::verify_drafts_sve2 and MTPHeads::generate_drafts
    wrappers (server/speculative_decoder.cpp:53-77, server/mtp_heads.cpp:53-79)
    around the C restatement of the Rust kernels they call.

Run from the repository root:  python tests/golden/gen_golden.py
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref.so")
OUT = os.path.join(ROOT, "tests", "golden", "ref_golden.npz")


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def main():
    subprocess.run(["bash", os.path.join(ROOT, "oracle", "build_ref.sh")], check=True)
    if not os.path.exists(LIB):
        sys.exit("reference library not built (reference tree missing)")
    L = C.CDLL(LIB)
    L.ref_kv_create.restype = C.c_void_p
    L.ref_kv_utilization.restype = C.c_float
    for fn in ("ref_kv_destroy", "ref_kv_append", "ref_kv_free_request", "ref_kv_share_prefix", "ref_kv_free_merged",
               "ref_kv_evict", "ref_kv_table", "ref_kv_utilization"):
        getattr(L, fn).argtypes = None
    rng = np.random.default_rng(20261201)
    data = {}

    # ---------------------------------------------- compute_paged_attention
    pa_cases = [(3, 8, 4, 12), (4, 16, 16, 9), (2, 32, 8, 6)]  # (M, hidden, block_size, pool_blocks)
    for ci, (M, H, bs, nblk) in enumerate(pa_cases):
        q = (rng.standard_normal((M, H)) * 0.5).astype(np.float32)
        kp = (rng.standard_normal((nblk * bs, H)) * 0.5).astype(np.float32)
        vp = rng.standard_normal((nblk * bs, H)).astype(np.float32)
        lens, tabs = [], []
        for m in range(M):
            sl = int(rng.integers(0, 3 * bs)) if m else 0  # request 0 has seq_len 0 (skipped)
            nb = (sl + bs - 1) // bs
            if m == M - 1 and sl > 0:
                nb += 1  # an extra trailing block beyond seq_len is ignored by the reference loop
            tabs.append(rng.choice(nblk, size=nb, replace=False).astype(np.int32))
            lens.append(sl)
        off = np.zeros(M + 1, np.int32)
        for m in range(M):
            off[m + 1] = off[m] + tabs[m].size
        flat = np.concatenate(tabs).astype(np.int32) if off[-1] else np.zeros(1, np.int32)
        lens = np.asarray(lens, np.int32)
        o = np.zeros((M, H), np.float32)
        L.ref_paged_attention(p(q), p(kp), p(vp), C.c_size_t(kp.size), p(off), p(flat), p(lens), p(o), M, H, bs)
        for name, arr in (("q", q), ("k", kp), ("v", vp), ("off", off), ("tables", flat), ("lens", lens), ("o", o)):
            data[f"pa{ci}_{name}"] = arr
        data[f"pa{ci}_shape"] = np.asarray([M, H, bs, nblk], np.int32)

    # ------------------------------------------------------ PagedKVCache
    num_blocks, bs, hid = 24, 16, 4
    h = C.c_void_p(L.ref_kv_create(num_blocks, bs, hid))
    ops = [("append", 0, 40), ("append", 1, 5), ("append", 2, 33), ("append", 0, 9), ("free", 1, 0),
           ("append", 3, 17), ("share", 4, 0, 35), ("append", 4, 20), ("merged", 2, 1), ("append", 1, 64),
           ("evict", 0, 20), ("append", 5, 200), ("append", 6, 3), ("free", 0, 0), ("append", 6, 50),
           ("merged", 4, 5), ("evict", 3, 1), ("append", 2, 31)]
    n_req = 7
    op_arr, tabs_after, lens_after, util_after, ret_after = [], [], [], [], []
    for op in ops:
        kind = op[0]
        ret = 0
        if kind == "append":
            ret = L.ref_kv_append(h, op[1], op[2], hid)
            op_arr.append([0, op[1], op[2], 0])
        elif kind == "free":
            L.ref_kv_free_request(h, op[1])
            op_arr.append([1, op[1], 0, 0])
        elif kind == "share":
            L.ref_kv_share_prefix(h, op[1], op[2], op[3])
            op_arr.append([2, op[1], op[2], op[3]])
        elif kind == "merged":
            L.ref_kv_free_merged(h, op[1], op[2])
            op_arr.append([3, op[1], op[2], 0])
        elif kind == "evict":
            ret = L.ref_kv_evict(h, op[1], op[2])
            op_arr.append([4, op[1], op[2], 0])
        t = np.full((n_req, 32), -1, np.int32)
        ln = np.zeros(n_req, np.int32)
        for r in range(n_req):
            buf = np.zeros(32, np.int32)
            lv = C.c_int32(0)
            n = L.ref_kv_table(h, r, p(buf), 32, C.byref(lv))
            t[r, :n] = buf[:n]
            ln[r] = lv.value
        tabs_after.append(t)
        lens_after.append(ln)
        util_after.append(L.ref_kv_utilization(h))
        ret_after.append(ret)
    L.ref_kv_destroy(h)
    data["kv_cfg"] = np.asarray([num_blocks, bs, hid, n_req], np.int32)
    data["kv_ops"] = np.asarray(op_arr, np.int32)
    data["kv_tables"] = np.stack(tabs_after)
    data["kv_lens"] = np.stack(lens_after)
    data["kv_util"] = np.asarray(util_after, np.float32)
    data["kv_ret"] = np.asarray(ret_after, np.int32)

    # ------------------------------------------- SpeculativeDecoder wrapper
    B, max_d, V = 5, 3, 40
    logits = rng.standard_normal((B, max_d, V)).astype(np.float32)
    drafts = np.zeros((B, max_d), np.int32)
    for b in range(B):
        for i in range(max_d):
            drafts[b, i] = int(np.argmax(logits[b, i])) if rng.random() < 0.6 else int(rng.integers(0, V))
    lens = np.asarray([3, 2, 0, 1, 3], np.int32)
    acc = np.zeros(B, np.int32)
    rep = np.zeros(B, np.int32)
    L.ref_verify(p(logits), C.c_size_t(logits.size), p(drafts), C.c_size_t(drafts.size), p(lens), B, V, max_d,
                 p(acc), p(rep))
    data.update(ver_logits=logits, ver_drafts=drafts, ver_lens=lens, ver_acc=acc, ver_rep=rep)

    # ---------------------------------------------------- MTPHeads wrapper
    K, H, V = 3, 16, 50
    W = (rng.standard_normal((K, H, V)) * 0.3).astype(np.float32)
    hs = rng.standard_normal(H).astype(np.float32)
    out = np.zeros(K, np.int32)
    L.ref_mtp_generate(p(W), p(hs), K, H, V, p(out))
    data.update(mtp_w=W, mtp_h=hs, mtp_out=out)

    np.savez_compressed(OUT, **data)
    print("wrote", OUT, sum(v.nbytes for v in data.values()), "bytes")


if __name__ == "__main__":
    main()
