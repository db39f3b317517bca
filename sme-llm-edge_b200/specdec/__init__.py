"""Host-side mirror of the sme-llm-edge speculative-decoding operator surface,
backed by libspecdec_sm100.so (CUDA, sm_100a).

The classes keep the reference's names and argument meanings:

  SpeculativeDecoder   server/speculative_decoder.h:12-35
  MTPHeads             server/mtp_heads.h:23-41
  compute_paged_attention  server/paged_attention.h:10-19
  PagedKVCache         server/paged_kv_cache.h:28-63

plus the device-resident step engine (`Engine`).  Every compute call runs a
CUDA kernel of libspecdec_sm100.so; there is no CPU path.  Importing this
module loads the library and raises if it is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# SPECDEC_LIB selects another build of the library (e.g. to compare two builds
# on one machine); the in-tree build otherwise.
LIB_PATH = os.environ.get("SPECDEC_LIB") or os.path.join(_HERE, "libspecdec_sm100.so")

OK, EINVAL, ENOMEM, ECUDA, ETIMEOUT, ENOTSUP, EFORMAT, EIO = range(8)


class SpecdecError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"specdec error {code}: {msg}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} not built; run `python sme-llm-edge_b200/build.py`")
    return C.CDLL(LIB_PATH)


_lib = _load()

P = C.c_void_p
I = C.c_int
F = C.c_float
SZ = C.c_size_t
U32 = C.c_uint32
U64 = C.c_uint64


class Sampling(C.Structure):
    _fields_ = [("temperature", F), ("top_p", F), ("seed", U64), ("step", U32)]


class ModelConfig(C.Structure):
    _fields_ = [("hidden", I), ("layers", I), ("n_q_heads", I), ("n_kv_heads", I), ("head_dim", I), ("ffn", I),
                ("vocab", I), ("n_mtp_heads", I), ("block_size", I), ("rms_eps", F), ("rope_theta", F)]


class SmeTensorView(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", U32), ("dims", C.POINTER(U32)), ("elements", U64),
                ("quantized", I), ("data_bytes", U32), ("scales", C.c_void_p), ("data", C.c_void_p)]


class RunConfig(C.Structure):
    _fields_ = [("batch", I), ("draft_len", I), ("tree_nodes", I), ("tree_branching", I * 8), ("tree_levels", I),
                ("max_ctx", I), ("num_blocks", I), ("use_graph", I), ("sampling", Sampling)]


_SIGS = {
    "specdec_last_error": (C.c_char_p, []),
    "specdec_abi_version": (I, []),
    "specdec_selftest_wait_timeout": (I, [P]),
    "sve2_speculative_verify_f32": (None, [P, P, P, U32, U32, U32, P, P]),
    "rust_sme_mtp_predict_f32": (None, [P, P, P, U32, U32, U32]),
    "rust_sme_mtp_sample_f32": (None, [P, P, U32, U32]),
    "specdec_compat_release_weights": (I, [C.POINTER(U64)]),
    "specdec_compat_weight_uploads": (I, [C.POINTER(U64)]),
    "sme_sm_prefetch_kv_blocks": (None, [P, P, U32]),
    "rust_sme_flashdecoding_chunk_f32": (None, [P, P, P, U32, U32, F, P, P, P]),
    "rust_sve2_flashdecoding_reduce_f32": (None, [P, P, P, U32, U32, P]),
    "specdec_paged_attention_compat_f32": (I, [P, P, P, SZ, P, P, P, P, I, I, I]),
    "specdec_accept_workspace_bytes": (SZ, [I]),
    "specdec_accept_chain": (I, [P, P, P, I, I, I, C.POINTER(Sampling), P, P, P, SZ, P]),
    "specdec_accept_chain_noalloc": (I, [P, P, P, I, I, I, C.POINTER(Sampling), P, P, P]),
    "specdec_accept_tree": (I, [P, P, P, I, I, I, C.POINTER(Sampling), P, P, P, P, SZ, P]),
    "specdec_sample_rows": (I, [P, I, I, I, C.POINTER(Sampling), P, P, SZ, P]),
    "specdec_compat_verify": (I, [P, P, P, I, I, I, P, P, P]),
    "specdec_shard_row_max": (I, [P, I, P, I, I, I, P, P, P]),
    "specdec_shard_merge_max": (I, [P, P, I, I, P, P, P]),
    "specdec_shard_row_mass": (I, [P, I, P, I, I, P, F, P, P]),
    "specdec_shard_digit_hist": (I, [P, I, P, I, I, P, F, P, I, P, P]),
    "specdec_shard_select_digit": (I, [P, I, I, P, F, P, P, P, P]),
    "specdec_shard_mass_hist": (I, [P, I, P, I, I, P, F, I, P, P, P, P]),
    "specdec_shard_cross": (I, [P, I, F, P, F, P, I, P, P, P, P]),
    "specdec_shard_union_select": (I, [P, I, I, P, P, F, P, P, P, P]),
    "specdec_shard_point_mass": (I, [P, P, P, I, I, I, I, F, P, P, P, P, P, P, P]),
    "specdec_shard_accept_test": (I, [P, I, I, C.POINTER(Sampling), P, P, P, P, P, P, P, P]),
    "specdec_shard_draw_winners": (I, [P, P, I, I, I, I, C.POINTER(Sampling), P, P, P, P, P, P, P, P, P, P]),
    "specdec_shard_draw_merge": (I, [P, I, I, I, P, P, P]),
    "specdec_w4_tiled_bytes": (SZ, [I, I]),
    "specdec_w4_tile": (I, [P, P, I, I, P, P]),
    "specdec_w4_untile": (I, [P, I, I, P, P, P]),
    "specdec_w4a16_workspace_bytes": (SZ, [I, I, I]),
    "specdec_w4a16_gemm": (I, [P, I, I, P, I, I, P, I, I, P, SZ, P]),
    "specdec_w4a16_gemm_swiglu": (I, [P, I, I, P, I, I, P, I, P]),
    "specdec_w4a16_gemv": (I, [P, I, I, P, I, I, P, I, I, P]),
    "specdec_w4a16_plan": (I, [I, I, I, I, P]),
    "specdec_w4a16_gemm_with_plan": (I, [P, I, I, P, I, I, P, I, I, I, I, P]),
    "specdec_w4a16_gemm_simt": (I, [P, I, I, P, I, I, P, I, I, P]),
    "specdec_attention_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "specdec_attention": (I, [P, P, I, I, I, P, I, P, P, I, I, I, P, P, SZ, P]),
    "specdec_kv_create": (I, [I, I, I, I, C.POINTER(P)]),
    "specdec_kv_destroy": (I, [P]),
    "specdec_kv_append": (I, [P, P, P, I, P, P]),
    "specdec_kv_free_request": (I, [P, I, P]),
    "specdec_kv_share_prefix": (I, [P, I, I, I, P]),
    "specdec_kv_free_merged_blocks": (I, [P, I, I, P]),
    "specdec_kv_evict_tokens": (I, [P, I, I, C.POINTER(I), P]),
    "specdec_kv_truncate": (I, [P, P, I, P]),
    "specdec_kv_utilization": (F, [P, P]),
    "specdec_kv_read": (I, [P, P, P, P, P]),
    "specdec_kv_tables_dev": (P, [P]),
    "specdec_kv_lens_dev": (P, [P]),
    "specdec_engine_create": (I, [C.POINTER(ModelConfig), C.POINTER(RunConfig), I, C.POINTER(P)]),
    "specdec_engine_destroy": (I, [P]),
    "specdec_engine_init_weights": (I, [P, U32]),
    "specdec_engine_load_sme": (I, [P, P, U32]),
    "specdec_engine_admit": (I, [P, I, C.c_int32, P, I, P, C.POINTER(C.c_int32)]),
    "specdec_engine_retire": (I, [P, I, P]),
    "specdec_engine_prefill_chunk": (I, [P, I, C.c_int32, P, I, I]),
    "specdec_engine_share_prefix": (I, [P, I, C.c_int32, P, I, P, C.POINTER(C.c_int32)]),
    "specdec_engine_draft": (I, [P]),
    "specdec_engine_verify_forward": (I, [P]),
    "specdec_engine_accept": (I, [P]),
    "specdec_engine_kv_commit_rollback": (I, [P]),
    "specdec_radix_create": (I, [C.POINTER(P)]),
    "specdec_radix_destroy": (I, [P]),
    "specdec_radix_match": (I, [P, P, I, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "specdec_radix_insert": (I, [P, C.c_int32, P, I]),
    "specdec_radix_release": (I, [P, C.c_int32]),
    "specdec_radix_stats": (I, [P, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "specdec_sme_open": (I, [C.c_char_p, C.POINTER(P)]),
    "specdec_sme_open_buffer": (I, [P, SZ, C.POINTER(P)]),
    "specdec_sme_close": (I, [P]),
    "specdec_sme_config_json": (I, [P, C.POINTER(C.c_char_p), C.POINTER(SZ)]),
    "specdec_sme_config_number": (I, [P, C.c_char_p, C.POINTER(C.c_double)]),
    "specdec_sme_vocab_size": (I, [P, C.POINTER(U32)]),
    "specdec_sme_token": (I, [P, U32, C.POINTER(C.c_void_p), C.POINTER(U32)]),
    "specdec_sme_token_id": (I, [P, C.c_char_p, U32, C.POINTER(C.c_int32)]),
    "specdec_sme_tensor_count": (I, [P, C.POINTER(U32)]),
    "specdec_sme_tensor_at": (I, [P, U32, C.POINTER(SmeTensorView)]),
    "specdec_sme_find": (I, [P, C.c_char_p, C.POINTER(SmeTensorView)]),
    "specdec_sme_model_config": (I, [P, C.POINTER(ModelConfig)]),
    "specdec_w4_convert": (I, [P, I, P, P, I, I, P, I, I, I, P]),
    "specdec_engine_prefill": (I, [P, P, I]),
    "specdec_engine_seed_state": (I, [P, P, U32]),
    "specdec_engine_step": (I, [P]),
    "specdec_engine_step_host": (I, [P, P, P]),
    "specdec_engine_set_active": (I, [P, P]),
    "specdec_engine_stream": (P, [P]),
    "specdec_engine_read": (I, [P, C.c_char_p, P, SZ]),
    "specdec_engine_write": (I, [P, C.c_char_p, P, SZ]),
    "specdec_engine_info": (I, [P, C.c_char_p, C.POINTER(C.c_int64)]),
    "specdec_engine_profile": (I, [P, I, P]),
    "specdec_engine_step_verify_timed": (I, [P, C.POINTER(F)]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED_SYMBOLS = tuple(_SIGS)


def lib():
    return _lib


def last_error() -> str:
    return (_lib.specdec_last_error() or b"").decode()


def check(rc: int):
    if rc != OK:
        raise SpecdecError(rc, last_error())


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def sampling(temperature: float, top_p: float = 1.0, seed: int = 0, step: int = 0) -> Sampling:
    return Sampling(float(temperature), float(top_p), int(seed), int(step))


# ======================================================================
# Reference operator surface
# ======================================================================
class ChunkedPrefillState:
    """server/chunked_prefill.h: a prompt handed out in chunks of
    `prefill_chunk_size` tokens (get_next_chunk, chunked_prefill.cpp:4-24),
    with the `advance_offset` the reference scheduler calls after a prefix
    match (continuous_scheduler.cpp:83).  Feed each chunk to
    Engine.prefill_chunk(seq, chunk, final=state.is_prefill_complete)."""

    def __init__(self, prompt_tokens=(), prefill_chunk_size: int = 64):
        self.prompt_tokens = [int(x) for x in prompt_tokens]
        self.prefill_chunk_size = int(prefill_chunk_size)
        self.prefill_offset = 0
        self.is_prefill_complete = False

    def get_next_chunk(self) -> list[int]:
        if self.is_prefill_complete or not self.prompt_tokens:
            return []
        n = min(len(self.prompt_tokens) - self.prefill_offset, self.prefill_chunk_size)
        chunk = self.prompt_tokens[self.prefill_offset:self.prefill_offset + n]
        self.prefill_offset += n
        if self.prefill_offset >= len(self.prompt_tokens):
            self.is_prefill_complete = True
        return chunk

    def get_remaining_tokens(self) -> int:
        return 0 if not self.prompt_tokens else len(self.prompt_tokens) - self.prefill_offset

    def reset(self):
        self.prefill_offset = 0
        self.is_prefill_complete = False

    def advance_offset(self, n: int):
        """Skips n prompt tokens already present (a shared prefix)."""
        self.prefill_offset = min(len(self.prompt_tokens), self.prefill_offset + int(n))
        if self.prompt_tokens and self.prefill_offset >= len(self.prompt_tokens):
            self.is_prefill_complete = True


class SpeculativeDecoder:
    """server/speculative_decoder.h: n-gram drafting on the host, verification on the GPU."""

    def __init__(self, max_draft: int = 3):
        self.max_draft_length = int(max_draft)
        self.ngram_table: dict[tuple[int, int], int] = {}

    def generate_draft(self, recent_tokens):
        # speculative_decoder.cpp:24-51 (bigram table lookup)
        out = []
        if len(recent_tokens) < 2:
            return out
        t1, t2 = int(recent_tokens[-2]), int(recent_tokens[-1])
        for _ in range(self.max_draft_length):
            nxt = self.ngram_table.get((t1, t2))
            if nxt is None:
                break
            out.append(nxt)
            t1, t2 = t2, nxt
        return out

    def update_ngram(self, t1: int, t2: int, next_token: int):
        self.ngram_table[(int(t1), int(t2))] = int(next_token)

    def verify_drafts_sve2(self, model_logits, draft_tokens, draft_lengths, vocab_size: int, batch_size: int):
        """speculative_decoder.cpp:53-77 -> sve2_speculative_verify_f32 on the GPU.

        model_logits is [batch, max_draft_length, vocab] (the decoder's own
        max_draft_length is the stride, as in the reference)."""
        acc = np.zeros(batch_size, np.int32)
        rep = np.full(batch_size, -1, np.int32)
        logits = np.ascontiguousarray(model_logits, dtype=np.float32).reshape(-1)
        drafts = np.ascontiguousarray(draft_tokens, dtype=np.int32).reshape(-1)
        lens = np.ascontiguousarray(draft_lengths, dtype=np.int32).reshape(-1)
        if logits.size == 0 or drafts.size == 0 or lens.size == 0:
            return acc, rep
        _lib.sve2_speculative_verify_f32(_p(logits), _p(drafts), _p(lens), vocab_size, self.max_draft_length,
                                         batch_size, _p(acc), _p(rep))
        return acc, rep


class MTPHeads:
    """server/mtp_heads.h: K draft heads of fp32 [K, hidden, vocab] weights."""

    def __init__(self, k_heads: int, hidden_dim: int, vocab_size: int):
        self.k_heads, self.hidden_dim, self.vocab_size = int(k_heads), int(hidden_dim), int(vocab_size)
        self.mtp_weights = np.zeros(self.k_heads * self.hidden_dim * self.vocab_size, np.float32)
        self.mtp_logits = np.zeros(self.k_heads * self.vocab_size, np.float32)

    def load_weights(self, weights_data):
        if weights_data is None:
            return
        self.mtp_weights[:] = np.asarray(weights_data, dtype=np.float32).reshape(-1)

    def generate_drafts(self, hidden_state):
        if hidden_state is None or not (self.hidden_dim and self.vocab_size and self.k_heads):
            return [-1] * self.k_heads
        h = np.ascontiguousarray(hidden_state, dtype=np.float32).reshape(-1)
        _lib.rust_sme_mtp_predict_f32(_p(h), _p(self.mtp_weights), _p(self.mtp_logits), self.hidden_dim,
                                      self.vocab_size, self.k_heads)
        out = np.zeros(self.k_heads, np.int32)
        _lib.rust_sme_mtp_sample_f32(_p(self.mtp_logits), _p(out), self.vocab_size, self.k_heads)
        return out.tolist()


def compute_paged_attention(batch_q, k_cache_pool, v_cache_pool, batch_block_tables, batch_seq_lens, batch_o,
                            hidden_dim: int, block_size: int):
    """server/paged_attention.cpp:16-111 semantics on the GPU; accumulates into batch_o (in place)."""
    q = np.ascontiguousarray(batch_q, dtype=np.float32).reshape(-1)
    kp = np.ascontiguousarray(k_cache_pool, dtype=np.float32).reshape(-1)
    vp = np.ascontiguousarray(v_cache_pool, dtype=np.float32).reshape(-1)
    M = len(batch_seq_lens)
    off = np.zeros(M + 1, np.int32)
    for m in range(M):
        off[m + 1] = off[m] + len(batch_block_tables[m])
    flat = np.zeros(max(1, int(off[-1])), np.int32)
    for m in range(M):
        flat[off[m]:off[m + 1]] = batch_block_tables[m]
    lens = np.ascontiguousarray(batch_seq_lens, dtype=np.int32)
    o = batch_o if isinstance(batch_o, np.ndarray) and batch_o.dtype == np.float32 else np.asarray(batch_o, np.float32)
    assert o.flags["C_CONTIGUOUS"]
    check(_lib.specdec_paged_attention_compat_f32(_p(q), _p(kp), _p(vp), kp.size, _p(off), _p(flat), _p(lens), _p(o),
                                                  M, hidden_dim, block_size))
    return o


class PagedKVCache:
    """server/paged_kv_cache.h: block tables kept in device memory.

    Allocation is lowest-free-index with reference counts, as the reference
    (paged_kv_cache.cpp:68-77); the K/V payload lives in the engine's fp16 pool."""

    def __init__(self, num_blocks: int, block_size: int, hidden_dim: int = 0, max_requests: int = 256,
                 max_blocks_per_request: int = 1024):
        self.num_blocks, self.block_size, self.hidden_dim = num_blocks, block_size, hidden_dim
        self.max_requests, self.max_bpr = max_requests, max_blocks_per_request
        h = P()
        check(_lib.specdec_kv_create(num_blocks, block_size, max_requests, max_blocks_per_request, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            _lib.specdec_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def append_tokens(self, request_id: int, n_tokens) -> int:
        """Appends tokens (a count, or K/V rows whose first dim is the count)."""
        n = int(n_tokens) if np.isscalar(n_tokens) else (np.asarray(n_tokens).size // max(1, self.hidden_dim))
        return self.append_batch([request_id], [n])[0]

    def append_batch(self, request_ids, n_tokens):
        reqs = np.ascontiguousarray(request_ids, dtype=np.int32)
        ns = np.ascontiguousarray(n_tokens, dtype=np.int32)
        last = np.zeros(reqs.size, np.int32)
        rc = _lib.specdec_kv_append(self._h, _p(reqs), _p(ns), reqs.size, _p(last), None)
        if rc not in (OK, ENOMEM):
            check(rc)
        return last.tolist()

    def get_cache_for_batch(self, request_ids):
        tabs, lens, _ = self.read()
        out_t, out_l = [], []
        for r in request_ids:
            row = tabs[r]
            out_t.append([int(x) for x in row[row >= 0]])
            out_l.append(int(lens[r]))
        return out_t, out_l

    def free_request(self, request_id: int):
        check(_lib.specdec_kv_free_request(self._h, request_id, None))

    def share_prefix(self, new_request_id: int, source_request_id: int, shared_length: int):
        check(_lib.specdec_kv_share_prefix(self._h, new_request_id, source_request_id, shared_length, None))

    def free_merged_blocks(self, request_id: int, num_blocks_to_free: int):
        check(_lib.specdec_kv_free_merged_blocks(self._h, request_id, num_blocks_to_free, None))

    def evict_least_important_blocks(self, request_id: int, num_tokens_to_evict: int) -> bool:
        ev = I(0)
        check(_lib.specdec_kv_evict_tokens(self._h, request_id, num_tokens_to_evict, C.byref(ev), None))
        return bool(ev.value)

    def truncate(self, new_lengths):
        nl = np.ascontiguousarray(new_lengths, dtype=np.int32)
        check(_lib.specdec_kv_truncate(self._h, _p(nl), nl.size, None))

    def get_utilization(self) -> float:
        return float(_lib.specdec_kv_utilization(self._h, None))

    def prefetch_kv_blocks(self, physical_block_indices):
        """No-op on the GPU (kept for interface parity with paged_kv_cache.cpp:156-176)."""
        return None

    def read(self):
        tabs = np.zeros((self.max_requests, self.max_bpr), np.int32)
        lens = np.zeros(self.max_requests, np.int32)
        refs = np.zeros(self.num_blocks, np.int32)
        check(_lib.specdec_kv_read(self._h, _p(tabs), _p(lens), _p(refs), None))
        return tabs, lens, refs


# ======================================================================
# Step engine
# ======================================================================
from model_shapes import MODEL_SHAPES  # noqa: E402  (sme-llm-edge_b200/model_shapes.py, pure Python)


class SmeTensor:
    """One tensor of a `.sme` file (the reference's Tensor, server/main.cpp:
    184-222): name, dims, is_quantized, row factors `scales` (f32 [dims[0]],
    127 / max|w| per row) and `data` (int8 or f32), as numpy views into the
    file mapping (valid while the SmeModel is open)."""

    def __init__(self, v: SmeTensorView):
        self.name = v.name.decode("utf-8", "replace")
        self.dims = tuple(int(v.dims[i]) for i in range(v.n_dims))
        self.is_quantized = bool(v.quantized)
        self.data_bytes = int(v.data_bytes)
        n = int(v.elements)
        if self.is_quantized:
            self.scales = np.frombuffer((C.c_char * (4 * self.dims[0])).from_address(v.scales), np.float32)
            self.data = np.frombuffer((C.c_char * n).from_address(v.data), np.int8) if n else np.zeros(0, np.int8)
        else:
            self.scales = None
            self.data = (np.frombuffer((C.c_char * (4 * n)).from_address(v.data), np.float32) if n
                         else np.zeros(0, np.float32))

    def dequantized(self) -> np.ndarray:
        """Weights as f32: q / scale per row for int8 tensors (the writer's
        definition, convert_model.py:8-23), the stored values otherwise."""
        if not self.is_quantized:
            return self.data.reshape(self.dims)
        q = self.data.reshape(self.dims[0], -1).astype(np.float32)
        return (q / self.scales[:, None]).reshape(self.dims)


class SmeModel:
    """A `.sme` model file (load_sme_model, server/main.cpp:112-228), parsed
    by the library's C++ loader over a read-only mapping of the file."""

    def __init__(self, path=None, buffer: bytes | None = None):
        h = P()
        if buffer is not None:
            self._buf = C.create_string_buffer(bytes(buffer), len(buffer)) if len(buffer) else None
            check(_lib.specdec_sme_open_buffer(self._buf, len(buffer), C.byref(h)))
        else:
            check(_lib.specdec_sme_open(os.fsencode(path), C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.specdec_sme_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    @property
    def config_json(self) -> str:
        p, n = C.c_char_p(), SZ(0)
        check(_lib.specdec_sme_config_json(self._h, C.byref(p), C.byref(n)))
        return C.string_at(p, n.value).decode("utf-8", "replace")

    def config_number(self, key: str):
        v = C.c_double(0)
        rc = _lib.specdec_sme_config_number(self._h, key.encode(), C.byref(v))
        return None if rc else v.value

    @property
    def vocab_size(self) -> int:
        n = U32(0)
        check(_lib.specdec_sme_vocab_size(self._h, C.byref(n)))
        return int(n.value)

    def token(self, i: int) -> bytes:
        p, n = C.c_void_p(), U32(0)
        check(_lib.specdec_sme_token(self._h, i, C.byref(p), C.byref(n)))
        return C.string_at(p, n.value) if n.value else b""

    def token_id(self, word) -> int:
        b = word.encode() if isinstance(word, str) else bytes(word)
        out = C.c_int32(0)
        check(_lib.specdec_sme_token_id(self._h, b, len(b), C.byref(out)))
        return int(out.value)

    def tensor_names(self) -> list:
        n = U32(0)
        check(_lib.specdec_sme_tensor_count(self._h, C.byref(n)))
        out = []
        for i in range(n.value):
            v = SmeTensorView()
            check(_lib.specdec_sme_tensor_at(self._h, i, C.byref(v)))
            out.append(v.name.decode("utf-8", "replace"))
        return out

    def tensor(self, name: str) -> SmeTensor:
        v = SmeTensorView()
        check(_lib.specdec_sme_find(self._h, name.encode(), C.byref(v)))
        return SmeTensor(v)

    def model_config(self) -> dict:
        mc = ModelConfig()
        check(_lib.specdec_sme_model_config(self._h, C.byref(mc)))
        return {f: getattr(mc, f) for f, _ in ModelConfig._fields_}


class RadixKVCache:
    """server/radix_kv_cache.h: prefix index of admitted prompts (host side,
    path-compressed, the reference's per-token semantics)."""

    def __init__(self):
        h = P()
        check(_lib.specdec_radix_create(C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.specdec_radix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def match_prefix(self, tokens):
        """-> (matched_token_count, source_request_id)"""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        m, src = C.c_int32(0), C.c_int32(-1)
        check(_lib.specdec_radix_match(self._h, _p(t), t.size, C.byref(m), C.byref(src)))
        return int(m.value), int(src.value)

    def insert_prefix(self, request_id: int, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(_lib.specdec_radix_insert(self._h, int(request_id), _p(t), t.size))

    def release_prefix(self, request_id: int):
        check(_lib.specdec_radix_release(self._h, int(request_id)))

    def stats(self):
        """-> (nodes, token positions) held by the tree."""
        n, p = C.c_int64(0), C.c_int64(0)
        check(_lib.specdec_radix_stats(self._h, C.byref(n), C.byref(p)))
        return int(n.value), int(p.value)


def model_config(shape: dict) -> ModelConfig:
    return ModelConfig(shape["hidden"], shape["layers"], shape["n_q_heads"], shape["n_kv_heads"], shape["head_dim"],
                       shape["ffn"], shape["vocab"], shape["n_mtp_heads"], 16, shape.get("rms_eps", 1e-5),
                       shape.get("rope_theta", 10000.0))


class Engine:
    """One GPU's speculative-decoding engine (weights, paged KV, step graph)."""

    def __init__(self, shape: dict, batch: int, draft_len: int = 4, max_ctx: int = 2048, temperature: float = 0.8,
                 top_p: float = 1.0, seed: int = 0, tree_branching=None, tree_nodes: int = 0, use_graph: bool = True,
                 device: int = 0, num_blocks: int = 0):
        self.shape = dict(shape)
        self.mc = model_config(shape)
        br = list(tree_branching or [])
        rc = RunConfig()
        rc.batch = batch
        rc.draft_len = draft_len
        rc.tree_nodes = tree_nodes
        for i, b in enumerate(br[:8]):
            rc.tree_branching[i] = b
        rc.tree_levels = len(br)
        rc.max_ctx = max_ctx
        rc.num_blocks = num_blocks
        rc.use_graph = 1 if use_graph else 0
        rc.sampling = sampling(temperature, top_p, seed, 0)
        self.rc = rc
        h = P()
        check(_lib.specdec_engine_create(C.byref(self.mc), C.byref(rc), device, C.byref(h)))
        self._h = h
        self.batch = batch
        self.rows = self.info("rows")
        self.draft_len = self.info("draft_len")

    def close(self):
        if getattr(self, "_h", None):
            _lib.specdec_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self, key: str) -> int:
        v = C.c_int64(0)
        check(_lib.specdec_engine_info(self._h, key.encode(), C.byref(v)))
        return int(v.value)

    def init_weights(self, seed: int):
        check(_lib.specdec_engine_init_weights(self._h, seed))

    def load_sme(self, model: "SmeModel", missing_seed: int = 0):
        """Weights from a `.sme` file (requantised to int4 group-128 on the
        device); MTP heads the file lacks are synthesised from missing_seed."""
        check(_lib.specdec_engine_load_sme(self._h, model.handle, missing_seed))

    @classmethod
    def from_sme(cls, path, batch: int, missing_seed: int = 0, **run):
        """Engine shaped by a `.sme` file's config, loaded with its weights."""
        with SmeModel(path) as m:
            shape = m.model_config()
            eng = cls(shape, batch, **run)
            eng.load_sme(m, missing_seed)
        return eng

    def prefill(self, prompts):
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        check(_lib.specdec_engine_prefill(self._h, _p(p), p.shape[1]))

    def admit(self, seq: int, request_id: int, prompt, cache: "RadixKVCache | None" = None) -> int:
        """Starts slot `seq` on a new request; with a prefix index, shares the
        KV blocks of an indexed prefix and prefills only the rest.  Returns
        the number of shared tokens."""
        p = np.ascontiguousarray(prompt, dtype=np.int32).reshape(-1)
        shared = C.c_int32(0)
        check(_lib.specdec_engine_admit(self._h, seq, int(request_id), _p(p), p.size,
                                        cache.handle if cache is not None else None, C.byref(shared)))
        return int(shared.value)

    def retire(self, seq: int, cache: "RadixKVCache | None" = None):
        check(_lib.specdec_engine_retire(self._h, seq, cache.handle if cache is not None else None))

    def share_prefix(self, seq: int, request_id: int, prompt, cache: "RadixKVCache | None" = None) -> int:
        """Starts slot `seq` on a new request for chunked admission: shares
        the indexed prefix (whole blocks) and returns the number of shared
        tokens; feed the rest with prefill_chunk (ChunkedPrefillState.
        advance_offset(shared)) and insert the prompt into the index when it
        is complete."""
        p = np.ascontiguousarray(prompt, dtype=np.int32).reshape(-1)
        shared = C.c_int32(0)
        check(_lib.specdec_engine_share_prefix(self._h, seq, int(request_id), _p(p), p.size,
                                               cache.handle if cache is not None else None, C.byref(shared)))
        return int(shared.value)

    def prefill_chunk(self, seq: int, tokens, final: bool, request_id: int = -1):
        """Feeds the next chunk of slot `seq`'s prompt (after a retire, the
        first chunk); with `final` the chunk's last token becomes the pending
        token.  See ChunkedPrefillState for the scheduler-side chunking."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        check(_lib.specdec_engine_prefill_chunk(self._h, seq, int(request_id), _p(t), t.size, int(bool(final))))

    def seed_state(self, ctx_len, seed: int):
        c = np.ascontiguousarray(ctx_len, dtype=np.int32)
        check(_lib.specdec_engine_seed_state(self._h, _p(c), seed))

    def step(self):
        check(_lib.specdec_engine_step(self._h))

    def draft(self):
        """Stage 1 of a step: drafted tokens (no host synchronisation)."""
        check(_lib.specdec_engine_draft(self._h))

    def verify_forward(self):
        """Stage 2: the verify forward over pending token + drafts."""
        check(_lib.specdec_engine_verify_forward(self._h))

    def accept(self):
        """Stage 3: acceptance -> read("accepted") / read("out_tokens")."""
        check(_lib.specdec_engine_accept(self._h))

    def kv_commit_rollback(self):
        """Stage 4: commit the accepted rows' K/V, roll the rest back."""
        check(_lib.specdec_engine_kv_commit_rollback(self._h))

    def step_host(self):
        acc = np.zeros(self.batch, np.int32)
        out = np.zeros((self.batch, self.rows), np.int32)
        check(_lib.specdec_engine_step_host(self._h, _p(acc), _p(out)))
        return acc, out

    def set_active(self, active):
        a = np.ascontiguousarray(active, dtype=np.int32)
        check(_lib.specdec_engine_set_active(self._h, _p(a)))

    def stream(self) -> int:
        return int(_lib.specdec_engine_stream(self._h) or 0)

    def read(self, what: str, dtype, shape):
        out = np.zeros(shape, dtype)
        check(_lib.specdec_engine_read(self._h, what.encode(), _p(out), out.nbytes))
        return out

    def profile(self, steps: int) -> dict:
        """Mean device ms per step by kernel category (eager steps, event after every launch)."""
        out = np.zeros(7, np.float32)
        check(_lib.specdec_engine_profile(self._h, steps, _p(out)))
        keys = ("gemm_verify", "attention", "gemm_draft", "accept", "other", "step", "verify_gemm_launches")
        return {k: float(v) for k, v in zip(keys, out)}

    def step_verify_timed(self) -> float:
        """One step (a graph with global-timer stamps around the verify
        forward); returns the verify forward's device ms."""
        v = F(0.0)
        check(_lib.specdec_engine_step_verify_timed(self._h, C.byref(v)))
        return float(v.value)

    def write(self, what: str, arr):
        a = np.ascontiguousarray(arr)
        check(_lib.specdec_engine_write(self._h, what.encode(), _p(a), a.nbytes))
