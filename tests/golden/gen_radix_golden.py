"""Generates tests/golden/radix_golden.npz by running the reference's own
RadixKVCache (server/radix_kv_cache.cpp, compiled unmodified by
oracle/build_ref.sh into oracle/_ref/libref.so) over a seeded script of
insert_prefix / release_prefix calls, recording match_prefix on a fixed set of
probe sequences after every call.

The script exercises shared prefixes, divergence in the middle of a run,
prefixes of earlier prompts, empty prompts, a second insert under a live id
(the reference replaces the remembered path without releasing the first),
releases of unknown ids and the removal of unreferenced subtrees.

Run from the repository root:  python tests/golden/gen_radix_golden.py
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref.so")
OUT = os.path.join(ROOT, "tests", "golden", "radix_golden.npz")


def script(seed=20261202, n_ops=160, n_probes=24):
    """(ops, probes): ops = [(kind 0 insert / 1 release, request id, tokens)]."""
    rng = np.random.default_rng(seed)
    bases = [rng.integers(0, 6, 40).tolist() for _ in range(4)]

    def prompt():
        b = bases[int(rng.integers(0, len(bases)))]
        cut = int(rng.integers(0, 36))
        tail = rng.integers(0, 6, int(rng.integers(0, 8))).tolist()
        return b[:cut] + tail

    ops = []
    live = set()
    for _ in range(n_ops):
        u = rng.random()
        if u < 0.55 or not live:
            req = int(rng.integers(0, 12))
            ops.append((0, req, prompt()))
            live.add(req)
        elif u < 0.9:
            req = int(rng.choice(sorted(live)))
            ops.append((1, req, []))
            live.discard(req)
        else:
            ops.append((1, int(rng.integers(50, 60)), []))  # an id never inserted
    probes = [prompt() for _ in range(n_probes - 2)] + [[], bases[0][:40]]
    return ops, probes


def pack(seqs):
    off = np.zeros(len(seqs) + 1, np.int64)
    off[1:] = np.cumsum([len(s) for s in seqs])
    flat = np.array([t for s in seqs for t in s], np.int32)
    return off, flat


def main():
    subprocess.run(["bash", os.path.join(ROOT, "oracle", "build_ref.sh")], check=True)
    if not os.path.exists(LIB):
        sys.exit("reference library not built (reference tree missing)")
    L = C.CDLL(LIB)
    L.ref_radix_create.restype = C.c_void_p
    L.ref_radix_destroy.argtypes = [C.c_void_p]
    L.ref_radix_insert.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]
    L.ref_radix_release.argtypes = [C.c_void_p, C.c_int]
    L.ref_radix_match.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    ops, probes = script()
    h = L.ref_radix_create()
    res = np.zeros((len(ops), len(probes), 2), np.int32)
    m, s = C.c_int32(), C.c_int32()
    for i, (kind, req, toks) in enumerate(ops):
        t = np.array(toks, np.int32)
        if kind == 0:
            L.ref_radix_insert(h, req, t.ctypes.data if t.size else None, t.size)
        else:
            L.ref_radix_release(h, req)
        for j, p in enumerate(probes):
            q = np.array(p, np.int32)
            L.ref_radix_match(h, q.ctypes.data if q.size else None, q.size, C.byref(m), C.byref(s))
            res[i, j] = (m.value, s.value)
    L.ref_radix_destroy(h)
    op_off, op_toks = pack([o[2] for o in ops])
    pr_off, pr_toks = pack(probes)
    np.savez_compressed(OUT, op_kind=np.array([o[0] for o in ops], np.int32),
                        op_req=np.array([o[1] for o in ops], np.int32), op_off=op_off, op_toks=op_toks,
                        probe_off=pr_off, probe_toks=pr_toks, results=res)
    print(f"wrote {OUT}: {len(ops)} calls x {len(probes)} probes")


if __name__ == "__main__":
    main()
