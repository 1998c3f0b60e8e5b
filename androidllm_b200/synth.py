"""Seeded random-init models in HF tensor naming, for tests and benchmarks.

Every tensor has its own generator ``default_rng([seed, index])``, so any
subset can be generated lazily, in any order or in parallel, and always gives
the same values.  Projections and embeddings are ``N(0, std)``; RMSNorm
weights are ``1 + 0.1 N(0, 1)`` so the norms are exercised with non-trivial
gains.
"""
import numpy as np

# Model shapes used by the tests and benchmarks (androidllm canon dicts,
# androidllm/config.py:34-48).
CANONS = {
    # toy Llama: hidden 256, 4 layers, 8 q / 2 kv heads, head_dim 32, FFN 688
    "toy": dict(model_type="llama", hidden=256, layers=4, heads=8, kv_heads=2, head_dim=32,
                intermediate=688, vocab=32000, rope_theta=10000.0, rms_eps=1e-6,
                max_len=2048, tied=True, name="toy-llama"),
    # Qwen2.5-1.5B shape
    "qwen2.5-1.5b": dict(model_type="qwen2", hidden=1536, layers=28, heads=12, kv_heads=2,
                         head_dim=128, intermediate=8960, vocab=151936, rope_theta=1e6,
                         rms_eps=1e-6, max_len=32768, tied=True, name="qwen2.5-1.5b-synth"),
    # Qwen2.5-0.5B shape (head_dim = 896 / 14 = 64)
    "qwen2.5-0.5b": dict(model_type="qwen2", hidden=896, layers=24, heads=14, kv_heads=2,
                         head_dim=64, intermediate=4864, vocab=151936, rope_theta=1e6,
                         rms_eps=1e-6, max_len=32768, tied=True, name="qwen2.5-0.5b-synth"),
    # Qwen2.5-7B shape
    "qwen2.5-7b": dict(model_type="qwen2", hidden=3584, layers=28, heads=28, kv_heads=4,
                       head_dim=128, intermediate=18944, vocab=152064, rope_theta=1e6,
                       rms_eps=1e-6, max_len=32768, tied=False, name="qwen2.5-7b-synth"),
}


def tensor_specs(canon):
    """[(hf_name, shape, kind)] in the order the shard writer consumes them."""
    h, nh, nkv, hd = canon["hidden"], canon["heads"], canon["kv_heads"], canon["head_dim"]
    inter, vocab = canon["intermediate"], canon["vocab"]
    specs = [("model.embed_tokens.weight", (vocab, h), "w")]
    for i in range(canon["layers"]):
        p = f"model.layers.{i}."
        specs += [
            (p + "self_attn.q_proj.weight", (nh * hd, h), "w"),
            (p + "self_attn.k_proj.weight", (nkv * hd, h), "w"),
            (p + "self_attn.v_proj.weight", (nkv * hd, h), "w"),
            (p + "self_attn.o_proj.weight", (h, nh * hd), "w"),
            (p + "mlp.gate_proj.weight", (inter, h), "w"),
            (p + "mlp.up_proj.weight", (inter, h), "w"),
            (p + "mlp.down_proj.weight", (h, inter), "w"),
            (p + "input_layernorm.weight", (h,), "norm"),
            (p + "post_attention_layernorm.weight", (h,), "norm"),
        ]
    specs.append(("model.norm.weight", (h,), "norm"))
    if not canon["tied"]:
        specs.append(("lm_head.weight", (vocab, h), "w"))
    return specs


def make_tensor(seed, index, shape, kind, std=0.02):
    rng = np.random.default_rng([int(seed), int(index)])
    if kind == "norm":
        return (1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)


def synth_tensors(canon, seed=0, std=0.02):
    """{hf_name: zero-arg callable returning the fp32 tensor}."""
    return {name: (lambda i=i, s=shape, k=kind: make_tensor(seed, i, s, k, std))
            for i, (name, shape, kind) in enumerate(tensor_specs(canon))}
