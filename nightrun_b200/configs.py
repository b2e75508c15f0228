"""Model-architecture presets for the seeded synthetic models.

Each preset is the `.nrm` v3 header metadata of one architecture
(crates/nr-model/src/format.rs:127-156) plus the synthetic-weight recipe
(`quant`: 0 = every linear weight Q8_0, 1 = Q4_K_M-style Q4_K/Q6_K mix with
Q6_K for token_embd/output and for attn_v/ffn_down in even layers).
`tied` = FLAG_TIED_EMBEDDINGS. `rope_freqs_tensor` = 1 writes a rope_freqs
factor tensor instead of the header's Llama-3 scaling (exercises
crates/nr-model/src/infer.rs:437-442).
"""
ARCH_LLAMA3, ARCH_QWEN3, ARCH_GRANITE = 1, 2, 3

_BASE = dict(ctx_train=131072, rope_factor=0.0, rope_low=0.0, rope_high=0.0, rope_orig_ctx=0.0,
             embed_scale=1.0, attn_scale=0.0, residual_scale=1.0, logit_scale=1.0,
             tied=1, rope_freqs_tensor=0)
_LLAMA3_ROPE = dict(rope_theta=500000.0, rope_factor=32.0, rope_low=1.0, rope_high=4.0,
                    rope_orig_ctx=8192.0)


def _cfg(**kw):
    c = dict(_BASE)
    c.update(kw)
    return c


CONFIGS = {
    # Config 0: Llama-3.2-1B architecture, every linear weight Q8_0.
    "llama1b_q8": _cfg(name="synthetic Llama-3.2-1B Q8_0", arch=ARCH_LLAMA3, dim=2048, n_layers=16,
                       n_heads=32, n_kv_heads=8, head_dim=64, ffn_dim=8192, vocab=128256,
                       norm_eps=1e-5, quant=0, **_LLAMA3_ROPE),
    # Config 2: Llama-3.2-3B architecture, Q4_K_M-style mix.
    "llama3b_q4km": _cfg(name="synthetic Llama-3.2-3B Q4_K_M", arch=ARCH_LLAMA3, dim=3072, n_layers=28,
                         n_heads=24, n_kv_heads=8, head_dim=128, ffn_dim=8192, vocab=128256,
                         norm_eps=1e-5, quant=1, **_LLAMA3_ROPE),
    # Config 3: Qwen3-4B architecture (per-head q/k RMSNorm, NEOX RoPE).
    "qwen3_4b_q4km": _cfg(name="synthetic Qwen3-4B Q4_K_M", arch=ARCH_QWEN3, dim=2560, n_layers=36,
                          n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=9728, vocab=151936,
                          norm_eps=1e-6, rope_theta=5000000.0, ctx_train=40960, quant=1),
    # Config 4: Granite-4.1-3B dense architecture with muP scalars.
    "granite3b_q4km": _cfg(name="synthetic Granite-4.1-3B Q4_K_M", arch=ARCH_GRANITE, dim=2560,
                           n_layers=40, n_heads=40, n_kv_heads=8, head_dim=64, ffn_dim=8192,
                           vocab=100352, norm_eps=1e-5, rope_theta=10000.0, quant=1,
                           embed_scale=12.0, attn_scale=0.015625, residual_scale=0.22, logit_scale=8.0),
    # Small models of each family for parity tests (seconds on the CPU oracle).
    "tiny_llama_q8": _cfg(name="tiny llama q8", arch=ARCH_LLAMA3, dim=256, n_layers=2, n_heads=4,
                          n_kv_heads=2, head_dim=64, ffn_dim=768, vocab=1000, norm_eps=1e-5, quant=0,
                          **_LLAMA3_ROPE),
    "tiny_llama_q4km": _cfg(name="tiny llama q4km", arch=ARCH_LLAMA3, dim=256, n_layers=2, n_heads=2,
                            n_kv_heads=1, head_dim=128, ffn_dim=512, vocab=1000, norm_eps=1e-5, quant=1,
                            tied=0, rope_freqs_tensor=1, rope_theta=500000.0),
    "tiny_qwen3": _cfg(name="tiny qwen3", arch=ARCH_QWEN3, dim=256, n_layers=2, n_heads=4, n_kv_heads=2,
                       head_dim=128, ffn_dim=768, vocab=1200, norm_eps=1e-6, rope_theta=5000000.0,
                       quant=1),
    "tiny_granite": _cfg(name="tiny granite", arch=ARCH_GRANITE, dim=256, n_layers=3, n_heads=4,
                         n_kv_heads=1, head_dim=64, ffn_dim=512, vocab=900, norm_eps=1e-5,
                         rope_theta=10000.0, quant=1, embed_scale=12.0, attn_scale=0.015625,
                         residual_scale=0.22, logit_scale=8.0),
}

# Seeds of the synthetic workloads (weights; prompt ids use seed + 1).
MODEL_SEED = 20251201


def prompt_ids(n, vocab, seed=MODEL_SEED + 1, hi=128000):
    """Seed-uniform token ids in [0, min(vocab, hi)) from a xorshift64 stream."""
    bound = min(vocab, hi)
    x = (seed | 1) & 0xFFFFFFFFFFFFFFFF
    out = []
    for _ in range(n):
        x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 7
        x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
        out.append((x >> 11) % bound)
    return out
