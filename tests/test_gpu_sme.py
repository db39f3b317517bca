"""GPU parity of `.sme` loading: the int4 group-128 converter and an engine
whose weights come from a model file.

  * specdec_w4_convert (int8 rows with row factors or f32 rows, an optional
    folded RMSNorm weight, plain / gate / up layouts, partial 128-column
    groups) is bit-exact with the oracle: values q / rs (times the fold) in
    float32, then the oracle's quantiser, then the tiled layout;
  * an engine loaded from the reference-written fixture holds bit-identical
    weights to the oracle's conversion of the same file (norms folded into
    q/k/v, gate/up, lm_head and the MTP head; embed_tokens as fp16 rows), and
    a prefill plus speculative steps match the oracle's forward over those
    weights (the step-engine tolerances);
  * a two-layer file in the Hugging Face naming, without lm_head (tied to the
    embedding) and without MTP heads (synthesised from the seed), loads into
    weights identical to the oracle's and steps in parity.
"""
import os

import numpy as np
import pytest

import oracle as O
import sme_format as SF
import specdec as S
from helpers import dev, interleave_gu, ptr, steps_match_oracle, stream_ptr, sync, tile_w4

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "tiny_llama.sme")

ROLE_NAMES = {
    "ref": dict(embed="embed_tokens", norm="norm", lm_head="lm_head", q="layers.{}.q_proj", k="layers.{}.k_proj",
                v="layers.{}.v_proj", o="layers.{}.o_proj", gate="layers.{}.gate_proj", up="layers.{}.up_proj",
                down="layers.{}.down_proj", attn_norm="layers.{}.attn_norm", ffn_norm="layers.{}.ffn_norm",
                mtp="mtp.{}.proj", mtp_norm="mtp.{}.norm"),
    "hf": dict(embed="model.embed_tokens.weight", norm="model.norm.weight", lm_head="lm_head.weight",
               q="model.layers.{}.self_attn.q_proj.weight", k="model.layers.{}.self_attn.k_proj.weight",
               v="model.layers.{}.self_attn.v_proj.weight", o="model.layers.{}.self_attn.o_proj.weight",
               gate="model.layers.{}.mlp.gate_proj.weight", up="model.layers.{}.mlp.up_proj.weight",
               down="model.layers.{}.mlp.down_proj.weight", attn_norm="model.layers.{}.input_layernorm.weight",
               ffn_norm="model.layers.{}.post_attention_layernorm.weight", mtp="mtp.{}.proj.weight",
               mtp_norm="mtp.{}.norm.weight"),
}


def _zero_tiled(N, K):
    return tile_w4(np.full((N, K // 2), 0x88, np.uint8), np.zeros((N, (K + 127) // 128), np.uint16), N, K)


@pytest.mark.parametrize("src,K,fold,layout", [
    ("int8", 4096, True, 0), ("f32", 4096, False, 0), ("int8", 200, True, 0), ("f32", 384, True, 1),
    ("int8", 256, False, 2), ("int8", 128, True, 1),
])
def test_w4_convert_matches_oracle(cuda_device, src, K, fold, layout):
    rng = np.random.default_rng(K + layout)
    F = 300  # rows per converted tensor (partial last 128-row unit)
    w = (rng.standard_normal((F, K)) * 0.03).astype(np.float32)
    w[7] = 0
    g = (1 + 0.2 * rng.standard_normal(K)).astype(np.float32) if fold else None
    if src == "int8":
        q, rs = SF.quantize_rows(w)
        t = dict(dims=(F, K), quantized=True, scales=rs, data=q.reshape(-1))
        d_src, d_rs = dev(q), dev(rs)
    else:
        t = dict(dims=(F, K), quantized=False, scales=None, data=w.reshape(-1))
        d_src, d_rs = dev(w), None
    p, s = O.w4_quantize(SF.sme_values(t, g))
    d_g = dev(g) if fold else None
    if layout == 0:
        N, row0 = 700, 211  # rows row0 .. row0 + F of a larger weight
        full_p = np.full((N, K // 2), 0x88, np.uint8)
        full_s = np.zeros((N, (K + 127) // 128), np.uint16)
        full_p[row0:row0 + F], full_s[row0:row0 + F] = p, s
        want = tile_w4(full_p, full_s, N, K)
    else:
        other = (np.full((F, K // 2), 0x88, np.uint8), np.zeros((F, (K + 127) // 128), np.uint16))
        gate, up = ((p, s), other) if layout == 1 else (other, (p, s))
        gp, gs, N = interleave_gu(gate, up, F)
        row0 = 0
        want = tile_w4(gp, gs, N, K)
    tiled = dev(_zero_tiled(N, K))
    assert tiled.numel() == S.lib().specdec_w4_tiled_bytes(N, K)
    S.check(S.lib().specdec_w4_convert(ptr(d_src), 1 if src == "f32" else 0, ptr(d_rs) if d_rs is not None else None,
                                       ptr(d_g) if fold else None, F, K, ptr(tiled), N, row0, layout, stream_ptr()))
    sync()
    np.testing.assert_array_equal(tiled.cpu().numpy(), want)


def _oracle_weights(raw: bytes, mc: dict, names: dict, missing_seed: int):
    """The oracle's conversion of a file: per-role packed / scales, fp16 embed."""
    f = SF.read_sme(raw)["tensors"]
    H, L, nm = mc["hidden"], mc["layers"], mc["n_mtp_heads"]

    def get(role, i=0):
        return f.get(names[role].format(i))

    def fold(role, i=0):
        t = get(role, i)
        return None if t is None else t["data"]

    def conv(role, i=0, g=None):
        return O.w4_quantize(SF.sme_values(get(role, i), g))

    proj = {r: [] for r in ("q", "k", "v", "o", "gate", "up", "down")}
    for l in range(L):
        for r in ("q", "k", "v"):
            proj[r].append(conv(r, l, fold("attn_norm", l)))
        proj["o"].append(conv("o", l))
        for r in ("gate", "up"):
            proj[r].append(conv(r, l, fold("ffn_norm", l)))
        proj["down"].append(conv("down", l))
    lm_t = get("lm_head") or get("embed")
    lm = O.w4_quantize(SF.sme_values(lm_t, fold("norm")))
    mtp = []
    for i in range(nm):
        if get("mtp", i) is not None:
            mtp.append(conv("mtp", i, fold("mtp_norm", i)))
        else:
            mtp.append(O.synth_w4(missing_seed, O.T_MTP0 + i, H, H))
    emb16 = O.f16_bits(SF.sme_values(get("embed")))
    return proj, lm, mtp, emb16


def _check_weights(eng, mc, proj, lm, mtp, emb16):
    H, F, V, hd = mc["hidden"], mc["ffn"], mc["vocab"], mc["head_dim"]
    qd, kd = mc["n_q_heads"] * hd, mc["n_kv_heads"] * hd
    tb = S.lib().specdec_w4_tiled_bytes
    for l in range(mc["layers"]):
        qkv = [proj[r][l] for r in ("q", "k", "v")]
        got = eng.read(f"w_qkv{l}", np.uint8, (tb(qd + 2 * kd, H),))
        np.testing.assert_array_equal(got, tile_w4(np.vstack([p for p, _ in qkv]), np.vstack([s for _, s in qkv]),
                                                   qd + 2 * kd, H), err_msg=f"qkv {l}")
        np.testing.assert_array_equal(eng.read(f"w_o{l}", np.uint8, (tb(H, qd),)), tile_w4(*proj["o"][l], H, qd))
        gp, gs, NGU = interleave_gu(proj["gate"][l], proj["up"][l], F)
        np.testing.assert_array_equal(eng.read(f"w_gu{l}", np.uint8, (tb(NGU, H),)), tile_w4(gp, gs, NGU, H))
        np.testing.assert_array_equal(eng.read(f"w_down{l}", np.uint8, (tb(H, F),)), tile_w4(*proj["down"][l], H, F))
    np.testing.assert_array_equal(eng.read("w_lm", np.uint8, (tb(V, H),)), tile_w4(*lm, V, H))
    for i, hw in enumerate(mtp):
        np.testing.assert_array_equal(eng.read(f"w_head{i}", np.uint8, (tb(H, H),)), tile_w4(*hw, H, H))
    np.testing.assert_array_equal(eng.read("emb", np.uint16, (V * H,)), emb16.reshape(-1))


def _run_parity(eng, model, mc, B, k, T, seed, prompt_len, steps):
    """Prefill, then speculative steps checked against the oracle."""
    rng = np.random.default_rng(seed)
    eng.prefill(rng.integers(0, mc["vocab"], (B, prompt_len)).astype(np.int32))
    steps_match_oracle(eng, model, mc, B, k, T, seed, steps)


@pytest.fixture(scope="module")
def fixture_raw():
    with open(FIXTURE, "rb") as f:
        return f.read()


def test_engine_from_reference_fixture(cuda_device, fixture_raw):
    with S.SmeModel(FIXTURE) as m:
        mc = m.model_config()
    proj, lm, mtp, emb16 = _oracle_weights(fixture_raw, mc, ROLE_NAMES["ref"], 0)
    eng = S.Engine.from_sme(FIXTURE, batch=2, draft_len=3, max_ctx=256, temperature=1.0, seed=3, use_graph=True)
    _check_weights(eng, mc, proj, lm, mtp, emb16)
    model = O.ArrayModel(mc, emb16, proj, lm, mtp, rope_max_pos=256 + 80)
    _run_parity(eng, model, mc, B=2, k=3, T=1.0, seed=3, prompt_len=90, steps=3)
    eng.close()


def test_engine_from_hf_named_file_tied_lm_synth_heads(cuda_device, tmp_path):
    H, L, Hq, Hkv, hd, F, V = 256, 2, 4, 2, 64, 384, 1000
    rng = np.random.default_rng(5)
    n = ROLE_NAMES["hf"]

    def w(*shape):
        return (rng.standard_normal(shape) * 0.03).astype(np.float32)

    def g():
        return (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)

    t = {n["embed"]: w(V, H)}
    for l in range(L):
        t.update({n["q"].format(l): w(Hq * hd, H), n["k"].format(l): w(Hkv * hd, H), n["v"].format(l): w(Hkv * hd, H),
                  n["o"].format(l): w(H, Hq * hd), n["gate"].format(l): w(F, H), n["up"].format(l): w(F, H),
                  n["down"].format(l): w(H, F), n["attn_norm"].format(l): g(), n["ffn_norm"].format(l): g()})
    t[n["norm"]] = g()
    cfg = {"model_type": "llama", "num_layers": L, "num_heads": Hq, "hidden_dim": H, "vocab_size": V,
           "num_key_value_heads": Hkv, "num_mtp_heads": 2, "max_seq_len": 2048}
    raw = SF.write_sme(cfg, [f"t{i}" for i in range(V)], t)
    path = tmp_path / "hf_tied.sme"
    path.write_bytes(raw)
    with S.SmeModel(str(path)) as m:
        mc = m.model_config()
    assert (mc["n_kv_heads"], mc["ffn"], mc["n_mtp_heads"]) == (Hkv, F, 2)
    proj, lm, mtp, emb16 = _oracle_weights(raw, mc, n, missing_seed=7)
    eng = S.Engine.from_sme(str(path), batch=1, missing_seed=7, draft_len=2, max_ctx=256, temperature=0.0, seed=1,
                            use_graph=False)
    _check_weights(eng, mc, proj, lm, mtp, emb16)
    model = O.ArrayModel(mc, emb16, proj, lm, mtp, rope_max_pos=256 + 80)
    _run_parity(eng, model, mc, B=1, k=2, T=0.0, seed=1, prompt_len=40, steps=2)
    eng.close()


def test_engine_load_rejects_mismatched_file(cuda_device, fixture_raw):
    with S.SmeModel(buffer=fixture_raw) as m:
        shape = m.model_config()
        shape["ffn"] = 256
        eng = S.Engine(shape, batch=1, draft_len=2, max_ctx=64, use_graph=False)
        with pytest.raises(S.SpecdecError) as e:
            eng.load_sme(m)
        assert e.value.code == S.EINVAL
        eng.close()
