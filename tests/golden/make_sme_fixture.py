"""Writes tests/golden/tiny_llama.sme with the reference's own writer.

The model (config, vocabulary, f32 tensors) comes from fixture_model(), seeded
and importable without the reference tree; the file is written by
save_sme_model from the reference's convert_model.py, imported from the
reference checkout (SME_LLM_EDGE_REF, default: `reference` beside the repo
root).  tests/test_sme.py checks the library's parser against this file and
checks the oracle's writer (oracle/sme_format.py) byte for byte against it.

    python tests/golden/make_sme_fixture.py
"""
import contextlib
import io
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "tiny_llama.sme")


def fixture_model():
    """One-layer Llama-shaped model in the reference's tensor names
    (convert_model.py:79-97) plus one MTP head and one small 2-D tensor that
    the writer stores as f32 (16 rows or fewer)."""
    rng = np.random.default_rng(20261202)
    H, F, V, hd, n_kv = 128, 128, 160, 64, 1
    config = {"model_type": "llama-sme-test", "num_layers": 1, "num_heads": 2, "hidden_dim": H, "vocab_size": V,
              "max_seq_len": 512}
    vocab = [f"<token_{i}>" for i in range(V)]
    vocab[:3] = ["<unk>", "<s>", "</s>"]
    for i, w in enumerate(["the", "local", "server", "runs", "llama", "model", "café", "算子"]):
        vocab[3 + i] = w

    def w(*shape, std=0.02):
        return (rng.standard_normal(shape) * std).astype(np.float32)

    t = {"embed_tokens": w(V, H)}
    t["layers.0.q_proj"] = w(2 * hd, H)
    t["layers.0.k_proj"] = w(n_kv * hd, H)
    t["layers.0.v_proj"] = w(n_kv * hd, H)
    t["layers.0.o_proj"] = w(H, 2 * hd)
    t["layers.0.gate_proj"] = w(F, H)
    t["layers.0.up_proj"] = w(F, H)
    t["layers.0.down_proj"] = w(H, F)
    t["layers.0.attn_norm"] = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    t["layers.0.ffn_norm"] = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    t["norm"] = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    t["lm_head"] = w(V, H)
    t["mtp.0.proj"] = w(H, H)
    t["mtp.0.norm"] = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    t["extra.small_f32"] = w(8, H)
    t["layers.0.q_proj"][5] = 0.0  # an all-zero row (row factor 1)
    return config, vocab, t


def main():
    ref = os.environ.get("SME_LLM_EDGE_REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "..",
                                                             "reference")
    sys.path.insert(0, os.path.abspath(ref))
    import convert_model  # the reference's writer

    config, vocab, tensors = fixture_model()
    with contextlib.redirect_stdout(io.StringIO()):
        convert_model.save_sme_model(OUT, config, vocab, tensors)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
