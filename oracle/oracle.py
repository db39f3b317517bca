"""ctypes bindings for the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: this module is the checker used by tests/, the
smoke() entry of __graft_entry__.py and the CPU-baseline legs of bench.py.
The product path (sme-llm-edge_b200) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I = C.c_int
U32 = C.c_uint32
U64 = C.c_uint64
F = C.c_float


class RowStats(C.Structure):
    _fields_ = [("max", C.c_float), ("tau", C.c_uint32), ("sum", C.c_uint64), ("nuc", C.c_uint64)]


class ModelCfg(C.Structure):
    _fields_ = [("hidden", I), ("layers", I), ("n_q_heads", I), ("n_kv_heads", I), ("head_dim", I), ("ffn", I),
                ("vocab", I), ("n_mtp_heads", I), ("block_size", I), ("rms_eps", F), ("rope_theta", F)]


class KVPool(C.Structure):
    _fields_ = [("layers", I), ("num_blocks", I), ("n_kv_heads", I), ("block_size", I), ("head_dim", I),
                ("pool", P)]


class Model(C.Structure):
    _fields_ = [("cfg", ModelCfg), ("emb", P), ("w_packed", P * 7), ("w_scales", P * 7), ("lm_packed", P),
                ("lm_scales", P), ("mtp_packed", P), ("mtp_scales", P), ("rope_cos", P), ("rope_sin", P),
                ("rope_max_pos", I), ("n_layers_present", I)]


def _declare(L):
    sig = {
        "orc_f32_to_f16": (C.c_uint16, [F]),
        "orc_f16_to_f32": (F, [C.c_uint16]),
        "orc_philox4x32_10": (None, [P, P, P]),
        "orc_exp2_fx31": (U32, [F]),
        "orc_logit_key": (U32, [F]),
        "orc_row_stats_compute": (None, [P, I, F, U64, C.POINTER(RowStats)]),
        "orc_row_mass": (U32, [P, C.POINTER(RowStats), F, I]),
        "orc_draw_row": (I, [P, I, F, C.POINTER(RowStats), U64, U32, U32, U32, U32, P, I]),
        "orc_det_log2": (F, [F]),
        "orc_neg_log2_uniform": (F, [U32]),
        "orc_gumbel_uniform": (U32, [U64, U32, U32, U32, U32, U32]),
        "orc_race_key": (F, [F, U32]),
        "orc_argmax": (I, [P, I]),
        "orc_topk": (None, [P, I, I, P]),
        "orc_uniform_u32": (U32, [U64, U32, U32, U32, U32]),
        "orc_uniform_u64": (U64, [U64, U32, U32, U32, U32]),
        "orc_accept_chain": (None, [P, P, P, I, I, I, F, F, U64, U32, P, P]),
        "orc_accept_tree": (None, [P, P, P, I, I, I, F, F, U64, U32, P, P, P]),
        "orc_sample_rows": (None, [P, I, I, I, F, F, U64, U32, P]),
        "orc_compat_argmax": (I, [P, I, I, I]),
        "orc_compat_verify": (None, [P, P, P, I, I, I, I, P, P]),
        "orc_compat_mtp_predict": (None, [P, P, P, I, I, I]),
        "orc_compat_mtp_sample": (None, [P, P, I, I, I]),
        "orc_compat_paged_attention": (None, [P, P, P, P, P, P, P, I, I, I]),
        "orc_flashdecoding_chunk": (None, [P, P, P, I, I, F, P, P, P]),
        "orc_flashdecoding_reduce": (None, [P, P, P, I, I, P]),
        "orc_synth_value": (F, [U32, U32, U64]),
        "orc_synth_w4": (None, [U32, U32, I, I, I, I, P, P]),
        "orc_synth_f16": (None, [U32, U32, U64, C.c_size_t, P]),
        "orc_w4_dequant": (None, [P, P, I, I, P]),
        "orc_w4_quantize": (None, [P, I, I, P, P]),
        "orc_w4a16_gemm": (None, [P, I, P, P, I, I, P, I, I]),
        "orc_rmsnorm_f16": (None, [P, P, I, F, P]),
        "orc_rope_tables": (None, [I, I, F, P, P]),
        "orc_attention": (None, [P, C.POINTER(KVPool), I, P, I, P, P, I, I, I, P]),
        "orc_model_create": (C.POINTER(Model), [C.POINTER(ModelCfg), U32, I, I]),
        "orc_model_free": (None, [C.POINTER(Model)]),
        "orc_forward": (None, [C.POINTER(Model), C.POINTER(KVPool), P, I, P, P, P, P, P, I, I, I, P, P]),
        "orc_draft_chain": (None, [C.POINTER(Model), P, I, I, F, F, U64, U32, P, P, P]),
        "orc_bm_create": (P, [I, I, I, I]),
        "orc_bm_free": (None, [P]),
        "orc_bm_append": (I, [P, I, I]),
        "orc_bm_free_request": (None, [P, I]),
        "orc_bm_share_prefix": (None, [P, I, I, I]),
        "orc_bm_free_tail_blocks": (None, [P, I, I]),
        "orc_bm_evict_tokens": (I, [P, I, I]),
        "orc_bm_truncate": (None, [P, I, I]),
        "orc_bm_utilization": (F, [P]),
        "orc_bm_table": (I, [P, I, P, I, P]),
        "orc_bm_refcount": (I, [P, I]),
        "orc_tree_build": (I, [P, I, I, P, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- helpers
def philox(ctr, key):
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    o = np.zeros(4, dtype=np.uint32)
    lib().orc_philox4x32_10(ptr(c), ptr(k), ptr(o))
    return o


U_ACCEPT, U_GUMBEL_DRAFT, U_GUMBEL_RESAMPLE = 1, 3, 4


def draw_row(z, temperature, top_p, seed, step, b, i, purpose=U_GUMBEL_DRAFT, exclude=()):
    """Draw (exponential race) from the nucleus distribution of row z (orc_draw_row)."""
    z = np.ascontiguousarray(z, dtype=np.float32)
    st = row_stats(z, temperature, top_p)
    ex = np.ascontiguousarray(exclude, dtype=np.int32) if len(exclude) else None
    return lib().orc_draw_row(ptr(z), z.size, temp_coeff(temperature), C.byref(st), seed, step, b, i, purpose,
                              ptr(ex) if ex is not None else None, 0 if ex is None else ex.size)


def temp_coeff(temperature: float) -> float:
    return float(np.float32(1.4426950408889634 / temperature))


def top_p_q32(top_p: float) -> int:
    if not top_p < 1.0:
        return 1 << 32
    return int(round(top_p * 4294967296.0))


def row_stats(z: np.ndarray, temperature: float, top_p: float = 1.0) -> RowStats:
    z = np.ascontiguousarray(z, dtype=np.float32)
    st = RowStats()
    lib().orc_row_stats_compute(ptr(z), z.size, temp_coeff(temperature), top_p_q32(top_p), C.byref(st))
    return st


def accept_chain(target, draft, drafts, temperature, top_p, seed, step):
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, k1, V = target.shape
    k = k1 - 1
    draft = np.ascontiguousarray(draft if draft is not None else np.zeros((B, k, V), np.float32), dtype=np.float32)
    drafts = np.ascontiguousarray(drafts, dtype=np.int32)
    acc = np.zeros(B, np.int32)
    out = np.zeros((B, k + 1), np.int32)
    lib().orc_accept_chain(ptr(target), ptr(draft), ptr(drafts), B, k, V, temperature, top_p, seed, step, ptr(acc),
                           ptr(out))
    return acc, out


def accept_tree(target, node_tokens, parent, temperature, top_p, seed, step):
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, R, V = target.shape
    node_tokens = np.ascontiguousarray(node_tokens, dtype=np.int32)
    parent = np.ascontiguousarray(parent, dtype=np.int32)
    acc = np.zeros(B, np.int32)
    path = np.zeros((B, R), np.int32)
    out = np.zeros((B, R), np.int32)
    lib().orc_accept_tree(ptr(target), ptr(node_tokens), ptr(parent), B, R, V, temperature, top_p, seed, step,
                          ptr(acc), ptr(path), ptr(out))
    return acc, path, out


def sample_rows(logits, k, temperature, top_p, seed, step):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, V = logits.reshape(-1, logits.shape[-1]).shape
    out = np.zeros(rows, np.int32)
    lib().orc_sample_rows(ptr(logits), rows, k, V, temperature, top_p, seed, step, ptr(out))
    return out


def compat_verify(logits, drafts, lens, vocab, max_draft, vl=4):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    drafts = np.ascontiguousarray(drafts, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    B = lens.size
    acc = np.zeros(B, np.int32)
    rep = np.zeros(B, np.int32)
    lib().orc_compat_verify(ptr(logits), ptr(drafts), ptr(lens), vocab, max_draft, B, vl, ptr(acc), ptr(rep))
    return acc, rep


def tree_build(branching, max_nodes):
    br = np.ascontiguousarray(branching, dtype=np.int32)
    parent = np.zeros(max_nodes, np.int32)
    depth = np.zeros(max_nodes, np.int32)
    rank = np.zeros(max_nodes, np.int32)
    anc = np.zeros(max_nodes, np.uint64)
    n = lib().orc_tree_build(ptr(br), br.size, max_nodes, ptr(parent), ptr(depth), ptr(rank), ptr(anc))
    return parent[:n].copy(), depth[:n].copy(), rank[:n].copy(), anc[:n].copy()


def synth_w4(seed, tid, N, K, n0=0, n=None):
    n = N if n is None else n
    packed = np.zeros((n, K // 2), np.uint8)
    scales = np.zeros((n, (K + 127) // 128), np.uint16)
    lib().orc_synth_w4(seed, tid, N, K, n0, n, ptr(packed), ptr(scales))
    return packed, scales


def w4_quantize(w):
    """int4 group-128 quantiser of the oracle generator over given f32 rows."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, K = w.shape
    packed = np.zeros((n, K // 2), np.uint8)
    scales = np.zeros((n, (K + 127) // 128), np.uint16)
    lib().orc_w4_quantize(ptr(w), n, K, ptr(packed), ptr(scales))
    return packed, scales


def w4_dequant(packed, scales):
    N, K2 = packed.shape
    out = np.zeros((N, K2 * 2), np.float32)
    lib().orc_w4_dequant(ptr(packed), ptr(scales), N, K2 * 2, ptr(out))
    return out


def w4a16_gemm(X16, packed, scales, Y=None, mode=0):
    X16 = np.ascontiguousarray(X16, dtype=np.uint16)
    M, K = X16.shape
    N = packed.shape[0]
    if Y is None:
        Y = np.zeros((M, N), np.float32)
    lib().orc_w4a16_gemm(ptr(X16), M, ptr(packed), ptr(scales), N, K, ptr(Y), Y.shape[1], mode)
    return Y


def f16_bits(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).astype(np.float16)).view(np.uint16)


def f16_vals(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------- model
def layer_tensor(layer: int, which: int) -> int:
    return layer * 16 + which


T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN = range(7)
T_EMB, T_LM, T_MTP0 = 0x10000, 0x10001, 0x10010


class OracleModel:
    """Synthetic W4A16 model held by the oracle (weights generated on the host)."""

    def __init__(self, cfg: dict, seed: int, n_layers_present: int = -1, rope_max_pos: int = 4096):
        self.cfg = cfg
        c = ModelCfg(cfg["hidden"], cfg["layers"], cfg["n_q_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn"],
                     cfg["vocab"], cfg["n_mtp_heads"], cfg.get("block_size", 16), cfg.get("rms_eps", 1e-5),
                     cfg.get("rope_theta", 10000.0))
        self._cfg = c
        self.m = lib().orc_model_create(C.byref(c), seed, n_layers_present, rope_max_pos)

    def close(self):
        if self.m:
            lib().orc_model_free(self.m)
            self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ArrayModel:
    """Oracle model over given weights (e.g. converted from a `.sme` file):
    emb fp16 bits [V, H]; proj = {name: [(packed, scales) per layer]} for
    q, k, v, o, gate, up, down; lm = (packed, scales); mtp = [(packed,
    scales)] per head.  Arrays are kept alive by this object."""

    _ORDER = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, cfg: dict, emb16, proj: dict, lm, mtp, rope_max_pos: int = 4096):
        self.cfg = cfg
        hd = cfg["head_dim"]
        self._keep = []

        def keep(a):
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a.ctypes.data

        c = ModelCfg(cfg["hidden"], cfg["layers"], cfg["n_q_heads"], cfg["n_kv_heads"], hd, cfg["ffn"], cfg["vocab"],
                     cfg["n_mtp_heads"], cfg.get("block_size", 16), cfg.get("rms_eps", 1e-5),
                     cfg.get("rope_theta", 10000.0))
        m = Model()
        m.cfg = c
        m.emb = keep(np.asarray(emb16, np.uint16))
        for i, name in enumerate(self._ORDER):
            m.w_packed[i] = keep(np.concatenate([p for p, _ in proj[name]]))
            m.w_scales[i] = keep(np.concatenate([sc for _, sc in proj[name]]))
        m.lm_packed, m.lm_scales = keep(lm[0]), keep(lm[1])
        m.mtp_packed = keep(np.concatenate([p for p, _ in mtp]))
        m.mtp_scales = keep(np.concatenate([sc for _, sc in mtp]))
        half = hd // 2
        cos_t = np.zeros((rope_max_pos, half), np.float32)
        sin_t = np.zeros((rope_max_pos, half), np.float32)
        lib().orc_rope_tables(rope_max_pos, hd, C.c_float(c.rope_theta), ptr(cos_t), ptr(sin_t))
        m.rope_cos, m.rope_sin = keep(cos_t), keep(sin_t)
        m.rope_max_pos = rope_max_pos
        m.n_layers_present = cfg["layers"]
        self._m = m
        self.m = C.pointer(m)

    def close(self):
        pass


class OracleKV:
    """Paged fp16 KV pool [L][blocks][2][Hkv][bs][hd] on the host."""

    def __init__(self, layers, num_blocks, n_kv_heads, block_size, head_dim):
        self.pool = np.zeros((layers, num_blocks, 2, n_kv_heads, block_size, head_dim), np.uint16)
        self.s = KVPool(layers, num_blocks, n_kv_heads, block_size, head_dim, self.pool.ctypes.data)


def forward(model: OracleModel, kv: OracleKV, tables, ctx_len, tokens, pos, slot, mask, B, R, n_layers=-1,
            want_logits=True, want_hidden=True):
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    ctx_len = np.ascontiguousarray(ctx_len, dtype=np.int32)
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    slot = np.ascontiguousarray(slot, dtype=np.int32)
    mask = np.ascontiguousarray(mask, dtype=np.uint64)
    M = B * R
    logits = np.zeros((M, model.cfg["vocab"]), np.float32) if want_logits else None
    hidden = np.zeros((M, model.cfg["hidden"]), np.float32) if want_hidden else None
    lib().orc_forward(model.m, C.byref(kv.s), ptr(tables), tables.shape[1], ptr(ctx_len), ptr(tokens), ptr(pos),
                      ptr(slot), ptr(mask), B, R, n_layers, ptr(logits) if logits is not None else None,
                      ptr(hidden) if hidden is not None else None)
    return logits, hidden


def draft_chain(model: OracleModel, h0, k, temperature, top_p, seed, step):
    h0 = np.ascontiguousarray(h0, dtype=np.float32)
    B = h0.shape[0]
    V, H = model.cfg["vocab"], model.cfg["hidden"]
    dl = np.zeros((B, k, V), np.float32)
    dr = np.zeros((B, k), np.int32)
    hid = np.zeros((B, k, H), np.float32)
    lib().orc_draft_chain(model.m, ptr(h0), B, k, temperature, top_p, seed, step, ptr(dl), ptr(dr), ptr(hid))
    return dl, dr, hid


class BlockManager:
    """Oracle restatement of PagedKVCache's block-table logic."""

    def __init__(self, num_blocks, block_size, max_reqs, max_blocks_per_req):
        self.h = lib().orc_bm_create(num_blocks, block_size, max_reqs, max_blocks_per_req)
        self.max_bpr = max_blocks_per_req
        self.num_blocks = num_blocks

    def __del__(self):
        try:
            lib().orc_bm_free(self.h)
        except Exception:
            pass

    def append(self, req, n):
        return lib().orc_bm_append(self.h, req, n)

    def free_request(self, req):
        lib().orc_bm_free_request(self.h, req)

    def share_prefix(self, new_req, src_req, shared_len):
        lib().orc_bm_share_prefix(self.h, new_req, src_req, shared_len)

    def free_tail_blocks(self, req, n):
        lib().orc_bm_free_tail_blocks(self.h, req, n)

    def evict_tokens(self, req, n):
        return bool(lib().orc_bm_evict_tokens(self.h, req, n))

    def truncate(self, req, new_len):
        lib().orc_bm_truncate(self.h, req, new_len)

    def utilization(self):
        return lib().orc_bm_utilization(self.h)

    def table(self, req):
        buf = np.zeros(self.max_bpr, np.int32)
        ln = C.c_int32(0)
        n = lib().orc_bm_table(self.h, req, ptr(buf), self.max_bpr, C.byref(ln))
        return buf[:n].tolist(), ln.value

    def refcounts(self):
        return [lib().orc_bm_refcount(self.h, b) for b in range(self.num_blocks)]
