"""Model shapes of the speculative-decoding workloads (pure Python: importing
this module loads no library, so CPU-only callers can use it).

  tiny       4 layers, hidden 512, 8 query / 2 KV heads (head dim 64), FFN 1376, vocab 32000
  llama3-8b  32 layers, hidden 4096, 32 / 8 heads (head dim 128), FFN 14336, vocab 128256
  14b        48 layers, hidden 5120, 40 / 8 heads (head dim 128), FFN 13824, vocab 152064

Each has 3 MTP draft heads (hidden -> hidden, sharing the lm_head).
"""

MODEL_SHAPES = {
    "tiny": dict(hidden=512, layers=4, n_q_heads=8, n_kv_heads=2, head_dim=64, ffn=1376, vocab=32000, n_mtp_heads=3),
    "llama3-8b": dict(hidden=4096, layers=32, n_q_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                      n_mtp_heads=3),
    "14b": dict(hidden=5120, layers=48, n_q_heads=40, n_kv_heads=8, head_dim=128, ffn=13824, vocab=152064,
                n_mtp_heads=3),
}
