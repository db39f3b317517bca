"""CPU checks of the C-ABI boundary: the library loads without a GPU and
exports every function declared in include/specdec.h."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "specdec.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = set()
    for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", src):
        name = m.group(1)
        if name in ("if", "sizeof", "defined", "extern"):
            continue
        names.add(name)
    return sorted(n for n in names if n.startswith(("specdec_", "sve2_", "rust_", "sme_")))


def test_library_exports_every_declared_symbol():
    import specdec

    out = subprocess.run(["nm", "-D", "--defined-only", specdec.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    assert len(declared_functions()) >= 40


def test_python_binding_covers_header():
    import specdec

    assert set(declared_functions()) <= set(specdec.EXPORTED_SYMBOLS)
    assert specdec.lib().specdec_abi_version() == 1


def test_invalid_arguments_fail_loudly_without_gpu():
    import ctypes as C

    import specdec

    rc = specdec.lib().specdec_w4a16_gemm(None, 4, 8, None, 8, 8, None, 8, 0, None, 0, None)
    assert rc == specdec.EINVAL and "bad argument" in specdec.last_error()
    h = C.c_void_p()
    assert specdec.lib().specdec_kv_create(0, 16, 1, 1, C.byref(h)) == specdec.EINVAL
    # the few-row contraction takes 0..64 rows and modes 0 / 1 only
    x = C.c_void_p(16)
    assert specdec.lib().specdec_w4a16_gemv(x, 65, 128, x, 128, 128, x, 128, 0, None) == specdec.EINVAL
    assert specdec.lib().specdec_w4a16_gemv(x, 4, 128, x, 128, 128, x, 128, 2, None) == specdec.EINVAL
    assert "0 <= M <= 64" in specdec.last_error()


def test_gemm_plan_is_consistent():
    """The planner's choice (host logic only): a valid token tile, units per
    CTA and split, and a grid of tiles x split; small weight matrices get
    one-unit tiles so the grid covers more SMs."""
    import ctypes as C

    import specdec

    out = (C.c_int32 * 4)()
    for M, N, K in [(1, 4096, 4096), (16, 4096, 4096), (160, 4096, 4096), (160, 4096, 14336), (160, 6144, 4096),
                    (160, 28672, 4096), (160, 128256, 4096), (300, 512, 256), (7, 100, 200)]:
        assert specdec.lib().specdec_w4a16_plan(M, N, K, 0, out) == 0
        MT, QN, S, grid = list(out)
        assert MT in (16, 32, 64, 128, 160) and (M <= MT or MT in (128, 160))
        assert QN in (1, 2) and S in (1, 2, 4, 8) and S <= (K + 127) // 128 and MT % S == 0
        m_tiles = (M + MT - 1) // MT
        n_tiles = (N + 128 * QN - 1) // (128 * QN)
        assert grid == m_tiles * n_tiles * S
    assert specdec.lib().specdec_w4a16_plan(160, 4096, 14336, 0, out) == 0 and out[1] == 1
    assert specdec.lib().specdec_w4a16_plan(160, 4096, 14336, 2, out) == 0 and out[1] == 2
    assert specdec.lib().specdec_w4a16_plan(0, 4096, 4096, 0, out) != 0


def test_shard_steps_reject_bad_arguments_without_gpu():
    """The vocabulary-sharded acceptance steps check shapes, ranks and
    pointers before touching the GPU."""
    import ctypes as C

    import specdec

    L = specdec.lib()
    dummy = C.c_void_p(16)
    sp = specdec.sampling(0.7, 0.9, 1, 0)
    # shard width 0 and above the 262144 limit
    assert L.specdec_shard_row_max(dummy, 4, None, 0, 0, 0, dummy, dummy, None) == specdec.EINVAL
    assert "shard width" in specdec.last_error()
    assert L.specdec_shard_row_mass(dummy, 4, None, 0, 262145, dummy, 0.7, dummy, None) == specdec.EINVAL
    # draft rows announced without a pointer
    assert L.specdec_shard_digit_hist(dummy, 4, None, 3, 128, dummy, 0.7, None, 3, dummy, None) == specdec.EINVAL
    # digits other than 0..3, a draft length of 0, and an empty world
    assert L.specdec_shard_select_digit(dummy, 4, 4, dummy, 0.9, dummy, dummy, dummy, None) == specdec.EINVAL
    assert L.specdec_shard_draw_winners(dummy, dummy, 2, 0, 128, 0, C.byref(sp), dummy, dummy, dummy, dummy, dummy,
                                        dummy, dummy, dummy, None, None) == specdec.EINVAL
    assert L.specdec_shard_draw_merge(dummy, 0, 2, 3, dummy, dummy, None) == specdec.EINVAL
    # the mass steps need a temperature
    assert L.specdec_shard_point_mass(dummy, dummy, dummy, 2, 3, 128, 0, 0.0, dummy, dummy, dummy, dummy, dummy,
                                      dummy, None) == specdec.EINVAL
