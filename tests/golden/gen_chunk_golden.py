"""Generates tests/golden/chunk_golden.npz by running the reference's own
ChunkedPrefillState (server/chunked_prefill.cpp, compiled unmodified by
oracle/build_ref.sh into oracle/_ref/libref.so) call by call: every
get_next_chunk over a set of prompt lengths and chunk sizes (empty prompt,
shorter than a chunk, exact multiples, one token over, chunk size 1, a
reset() in the middle), recording per call the chunk length, its first token,
get_remaining_tokens() and is_prefill_complete.

Run from the repository root:  python tests/golden/gen_chunk_golden.py
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref.so")
OUT = os.path.join(ROOT, "tests", "golden", "chunk_golden.npz")
CAP = 64

# (prompt length, chunk size, reset after call index or -1)
CASES = [(0, 64, -1), (1, 64, -1), (63, 64, -1), (64, 64, -1), (65, 64, -1), (200, 64, -1), (200, 50, -1),
         (7, 1, -1), (130, 64, 0), (130, 64, 1), (5, 8, 0)]


def main():
    if not os.path.exists(LIB):
        subprocess.run(["bash", os.path.join(ROOT, "oracle", "build_ref.sh")], check=True)
    lib = C.CDLL(LIB)
    lib.ref_chunked_prefill.restype = C.c_int
    lib.ref_chunked_prefill.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int]
    cases, records, ncalls = [], [], []
    for n, chunk, reset_after in CASES:
        toks = (np.arange(n, dtype=np.int32) * 7 + 3).astype(np.int32)
        out = np.full((CAP, 4), -9, np.int32)
        k = lib.ref_chunked_prefill(toks.ctypes.data_as(C.c_void_p), n, chunk, reset_after,
                                    out.ctypes.data_as(C.c_void_p), CAP)
        cases.append((n, chunk, reset_after))
        records.append(out)
        ncalls.append(k)
    np.savez(OUT, cases=np.array(cases, np.int32), records=np.stack(records), ncalls=np.array(ncalls, np.int32))
    print("wrote", OUT, "calls", ncalls)


if __name__ == "__main__":
    main()
