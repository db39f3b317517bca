"""`.sme` model files: the library's C++ parser against the reference's format.

Pins (CPU only; the parser touches no GPU):
  * the oracle's writer (oracle/sme_format.py) reproduces, byte for byte, the
    fixture written by the reference's save_sme_model (convert_model.py:26-67;
    tests/golden/make_sme_fixture.py);
  * the library parses that fixture into the same config, vocabulary and
    tensors (dims, quantisation flag, data size, row factors, data) as the
    oracle's reader (load_sme_model, server/main.cpp:112-228);
  * every truncation of the fixture is rejected with SPECDEC_EFORMAT, as is a
    bad magic header or a tensor larger than the file; trailing bytes are
    ignored and a repeated name replaces the earlier tensor (main.cpp:222);
  * tokenize_word's rule: unknown words map to id 1 (main.cpp:230-233);
  * the engine model config derived from the file (both naming schemes);
  * the oracle's int4 group-128 quantiser against a numpy restatement.
"""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import oracle as O
import specdec as S
import sme_format as SF

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "tiny_llama.sme")


def _fixture_model():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_sme_fixture", os.path.join(HERE, "golden",
                                                                                    "make_sme_fixture.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.fixture_model()


@pytest.fixture(scope="module")
def raw():
    with open(FIXTURE, "rb") as f:
        return f.read()


def test_oracle_writer_reproduces_reference_written_fixture(raw):
    config, vocab, tensors = _fixture_model()
    assert SF.write_sme(config, vocab, tensors) == raw


def test_parser_matches_oracle_reader(raw):
    ref = SF.read_sme(raw)
    with S.SmeModel(FIXTURE) as m:
        assert m.config_json == ref["config"]
        assert m.vocab_size == len(ref["vocab"])
        assert [m.token(i) for i in range(m.vocab_size)] == ref["vocab"]
        assert m.tensor_names() == list(ref["tensors"])
        for name, t in ref["tensors"].items():
            got = m.tensor(name)
            assert got.dims == t["dims"] and got.is_quantized == t["quantized"], name
            assert got.data_bytes == t["data_bytes"], name
            np.testing.assert_array_equal(got.data, t["data"], err_msg=name)
            if t["quantized"]:
                np.testing.assert_array_equal(got.scales, t["scales"], err_msg=name)
        assert m.config_number("num_layers") == 1 and m.config_number("hidden_dim") == 128
        assert m.config_number("no_such_key") is None
        # the f32 2-D tensor (16 rows or fewer) and the writer's int8 rows
        small = m.tensor("extra.small_f32")
        assert not small.is_quantized and small.dims == (8, 128)
        _, _, tensors = _fixture_model()
        np.testing.assert_array_equal(small.dequantized(), tensors["extra.small_f32"])
        q = m.tensor("layers.0.q_proj")
        assert q.scales[5] == 1.0 and not q.data.reshape(q.dims)[5].any()  # the all-zero row
        err = np.abs(q.dequantized() - tensors["layers.0.q_proj"]).max(axis=1)
        assert np.all(err <= 0.5 / q.scales + 1e-9)  # q / rs within half a step of w


def test_tokenize_word_rule(raw):
    with S.SmeModel(buffer=raw) as m:
        assert m.token_id("the") == 3 and m.token_id("café") == 9 and m.token_id("算子") == 10
        assert m.token_id("<unk>") == 0 and m.token_id("</s>") == 2
        assert m.token_id("never-seen") == 1 and m.token_id("") == 1


def test_every_truncation_is_rejected(raw):
    buf = C.create_string_buffer(raw, len(raw))
    h = C.c_void_p()
    L = S.lib()
    for cut in range(len(raw)):
        rc = L.specdec_sme_open_buffer(buf, cut, C.byref(h))
        assert rc == S.EFORMAT and not h.value, cut
    assert L.specdec_sme_open_buffer(buf, len(raw), C.byref(h)) == S.OK
    L.specdec_sme_close(h)


def test_malformed_headers(raw):
    for bad in (b"", b"SME_MODE", b"XME_MODEL" + raw[9:], b"sme_model" + raw[9:]):
        with pytest.raises(S.SpecdecError) as e:
            S.SmeModel(buffer=bad)
        assert e.value.code == S.EFORMAT
    # a tensor whose element count exceeds the file
    hdr = SF.write_sme({"num_layers": 1}, ["a"], {})[:-4]
    big = hdr + struct.pack("<I", 1) + struct.pack("<I", 1) + b"x" + struct.pack("<III", 2, 0xFFFFFFFF, 0xFFFFFFFF)
    big += b"\x01" + struct.pack("<I", 0)
    with pytest.raises(S.SpecdecError) as e:
        S.SmeModel(buffer=big)
    assert e.value.code == S.EFORMAT
    with pytest.raises(S.SpecdecError) as e:
        S.SmeModel(os.path.join(HERE, "golden", "no_such_file.sme"))
    assert e.value.code == S.EIO


def test_trailing_bytes_and_repeated_names(raw):
    with S.SmeModel(buffer=raw + b"\0" * 37) as m:
        assert len(m.tensor_names()) == 15
    a = np.arange(40 * 8, dtype=np.float32).reshape(40, 8) / 100
    b = -a[:20]
    blob = SF.write_sme({"num_layers": 1}, ["x"], {"w": a, "v": np.ones(3, np.float32)})
    # second "w" appended by hand: tensor count 3, the later one wins
    extra = SF.write_sme({}, [], {"w": b})
    extra_tensor = extra[extra.index(b"w") - 4:]
    cnt_at = blob.index(struct.pack("<I", 2) + struct.pack("<I", 1) + b"w")
    blob2 = blob[:cnt_at] + struct.pack("<I", 3) + blob[cnt_at + 4:] + extra_tensor
    ref = SF.read_sme(blob2)
    with S.SmeModel(buffer=blob2) as m:
        assert m.tensor_names() == ["w", "v"]
        w = m.tensor("w")
        assert w.dims == (20, 8)
        np.testing.assert_array_equal(w.data, ref["tensors"]["w"]["data"])


def test_model_config_from_file(raw):
    with S.SmeModel(buffer=raw) as m:
        mc = m.model_config()
    assert (mc["hidden"], mc["layers"], mc["n_q_heads"], mc["n_kv_heads"], mc["head_dim"], mc["ffn"], mc["vocab"],
            mc["n_mtp_heads"]) == (128, 1, 2, 1, 64, 128, 160, 1)
    assert abs(mc["rms_eps"] - 1e-5) < 1e-12 and mc["rope_theta"] == 10000.0
    # Hugging Face names, explicit config keys, no MTP heads
    H, hd = 256, 64
    rng = np.random.default_rng(0)
    t = {"model.embed_tokens.weight": rng.standard_normal((300, H)).astype(np.float32),
         "model.layers.0.self_attn.k_proj.weight": rng.standard_normal((128, H)).astype(np.float32),
         "model.layers.0.mlp.gate_proj.weight": rng.standard_normal((384, H)).astype(np.float32)}
    cfg = {"num_layers": 2, "num_heads": 4, "hidden_dim": H, "vocab_size": 300, "num_kv_heads": 2,
           "rope_theta": 500000.0, "rms_norm_eps": 1e-6, "num_mtp_heads": 2}
    with S.SmeModel(buffer=SF.write_sme(cfg, ["a"], t)) as m:
        mc = m.model_config()
    assert (mc["n_kv_heads"], mc["head_dim"], mc["ffn"], mc["n_mtp_heads"], mc["rope_theta"]) == (2, hd, 384, 2,
                                                                                                    500000.0)
    assert abs(mc["rms_eps"] - 1e-6) < 1e-12
    # a file without the required projections is rejected
    with S.SmeModel(buffer=SF.write_sme({"num_layers": 1}, [], {})) as m:
        with pytest.raises(S.SpecdecError) as e:
            m.model_config()
        assert e.value.code == S.EFORMAT


def _np_w4_quantize(w):
    """numpy restatement: s = fp16(amax / 7) per 128 columns (1 when amax = 0),
    q = clamp(round-half-away(w / s), -8, 7), u4 = q + 8, low nibble = even k."""
    n, K = w.shape
    G = (K + 127) // 128
    packed = np.zeros((n, K // 2), np.uint8)
    scales = np.zeros((n, G), np.uint16)
    for g in range(G):
        wg = w[:, 128 * g:128 * g + 128]
        amax = np.abs(wg).max(axis=1)
        s16 = (amax / np.float32(7)).astype(np.float16)
        s16[amax == 0] = np.float16(1)
        scales[:, g] = s16.view(np.uint16)
        x = (wg / s16.astype(np.float32)[:, None]).astype(np.float64)
        q = np.clip(np.trunc(x + np.copysign(0.5, x)), -8, 7).astype(np.int64) + 8
        packed[:, 64 * g:64 * g + wg.shape[1] // 2] = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return packed, scales


@pytest.mark.parametrize("K", [128, 200, 384])
def test_oracle_quantizer_matches_numpy(K):
    rng = np.random.default_rng(K)
    w = (rng.standard_normal((37, K)) * 0.05).astype(np.float32)
    w[3] = 0
    w[4, :7] = [0.5, -0.5, 1.5, 7.5, -7.5, 3.4999998, 2.5000002]  # ties and near-ties at s = 1 after scaling
    p, s = O.w4_quantize(w)
    pn, sn = _np_w4_quantize(w)
    np.testing.assert_array_equal(s, sn)
    np.testing.assert_array_equal(p, pn)
