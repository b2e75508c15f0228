"""Tensor-parallel partition of a model over n ranks (the rule the library's
nrc_tp_ctx_new applies; nrc_tp_shard reports it for a live context).

Each rank computes whole output rows with the full K: query heads and KV
heads by whole KV groups (GQA groups never straddle ranks), and equal
contiguous row ranges of wo / ffn_down (model dim), ffn_gate / ffn_up (ffn)
and the classifier (vocabulary). Ranks then all-gather activations, never
partial sums, so every value is computed exactly as on one GPU.
"""


def shard(meta, n, r):
    """(nranks, rank, q head0, q heads, kv head0, kv heads, dim row0, dim rows,
    ffn row0, ffn rows, vocab row0, vocab rows) of rank r; meta is a dict with
    n_heads, n_kv_heads, dim, ffn_dim, vocab. Raises ValueError when the
    model does not split evenly."""
    if not (1 <= n and 0 <= r < n):
        raise ValueError(f"rank {r} of {n}")
    for k in ("n_kv_heads", "dim", "ffn_dim", "vocab"):
        if meta[k] % n:
            raise ValueError(f"{k}={meta[k]} does not split over {n} ranks")
    gqa = meta["n_heads"] // meta["n_kv_heads"]
    nkv = meta["n_kv_heads"] // n
    dn, fn, vn = meta["dim"] // n, meta["ffn_dim"] // n, meta["vocab"] // n
    return (n, r, r * nkv * gqa, nkv * gqa, r * nkv, nkv, r * dn, dn, r * fn, fn, r * vn, vn)
