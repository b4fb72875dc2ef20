"""The workloads, as synthetic-model specs (ssfgen_spec fields).

Shapes follow the five benchmark configurations: a Qwen2.5-1.5B-shaped dense
decoder (Q4), a GEMV microbench at 4096/14336 (Q4 and Q8), a Qwen3-30B-A3B-
shaped MoE layer, a Llama-3-8B-shaped decoder with 6-bit group fields, and a
Qwen3-235B-A22B-shaped MoE decoder. Weights are seeded N(0, 0.02) quantized
round-to-nearest; norms are 1.
"""

_BASE = dict(rope_theta=1e6, rms_eps=1e-6, tied=0, qkv_bias=0, qk_norm=0, nbits=4, emb_nbits=4,
             scale6=0, minneg=0, n_expert=0, n_expert_used=0, moe_flags=0, expert_ff=0,
             perm_mode=1, seed=1234, sigma=0.02, threads=0, direct=0)

CONFIGS = {
    # 0: Qwen2.5-1.5B shape, v8 Q4, tied head, q/k/v biases
    "qwen2.5-1.5b-q4": dict(_BASE, n_layer=28, n_embd=1536, n_head=12, n_head_kv=2, head_dim=128,
                            n_ff=8960, n_vocab=151936, tied=1, qkv_bias=1),
    # 1: GEMV shapes (attn_q 4096x4096, ffn_gate/up 14336x4096, ffn_down 4096x14336)
    "gemv-4096-q4": dict(_BASE, n_layer=1, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128,
                         n_ff=14336, n_vocab=1024),
    "gemv-4096-q8": dict(_BASE, n_layer=1, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128,
                         n_ff=14336, n_vocab=1024, nbits=8, emb_nbits=8),
    # 2: Qwen3-30B-A3B MoE layer shape
    "qwen3-30b-a3b-moe-layer": dict(_BASE, n_layer=1, n_embd=2048, n_head=32, n_head_kv=4, head_dim=128,
                                    n_ff=768, n_vocab=1024, n_expert=128, n_expert_used=8, moe_flags=1,
                                    expert_ff=768, qk_norm=1),
    # 3: Llama-3-8B shape, v9 6-bit fields ("Q4_K-style")
    "llama3-8b-q4k": dict(_BASE, n_layer=32, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128,
                          n_ff=14336, n_vocab=128256, rope_theta=5e5, rms_eps=1e-5, scale6=1, minneg=1),
    # 4: Qwen3-235B-A22B shape: 94 MoE layers, 64/4 heads with Q/K norm, 128
    # experts top-8 (softmax, renormalised), expert FFN 1536, untied head;
    # ~136 GB of Q4: codes and group ranges drawn directly, and the experts'
    # bytes (97 %) left out of the file for the engine to draw on the device
    # (sb_draw_experts); direct=1 writes them (shallow parity models)
    "qwen3-235b-a22b-q4": dict(_BASE, n_layer=94, n_embd=4096, n_head=64, n_head_kv=4, head_dim=128,
                               n_ff=1536, n_vocab=151936, n_expert=128, n_expert_used=8, moe_flags=1,
                               expert_ff=1536, qk_norm=1, direct=2),
}

# Small models for parity tests (same code paths, seconds on the CPU oracle).
TEST_CONFIGS = {
    "tiny-q4": dict(_BASE, n_layer=2, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, n_ff=512,
                    n_vocab=1024, qkv_bias=1),
    "small-q4-tied": dict(_BASE, n_layer=4, n_embd=512, n_head=8, n_head_kv=2, head_dim=64, n_ff=1408,
                          n_vocab=4096, tied=1, qkv_bias=1),
}


def spec_for(name, **over):
    """A copy of a named spec with overrides."""
    src = CONFIGS.get(name) or TEST_CONFIGS[name]
    s = dict(src)
    s.update(over)
    return s
