"""The benchmark-shape parity cases behind qwen.npz, shared by the script that
generates the fixture from the reference (make_golden.py) and the tests.

Two 2-layer models with the benchmark's layer shapes: a Qwen2.5-1.5B-shaped
target (hidden 1536, 12/2 heads, head_dim 128, FFN 8960, int4 attention, int8
MLP, tied int8 per-row 151936-row head) and a Qwen2.5-0.5B-shaped draft
(hidden 896, 14/2 heads, head_dim 64, FFN 4864, int4, tied int8 head).  Before
each case the KV cache of positions 0..QWEN_FILL-1 of every layer is filled
with seeded fp16 values, so a single forward at position 511-771 attends over
the context lengths of the benchmark's episode without a 700-token prefill.
"""
import numpy as np

from androidllm_b200 import synth

# (name, canon, seed, shard kwargs)
QWEN_MODELS = [
    ("qwen_t", dict(synth.CANONS["qwen2.5-1.5b"], layers=2, max_len=1024, name="qwen1.5b-2l"), 21,
     dict(attn_bits=4, mlp_bits=8, block=64, embed_bits=8)),
    ("qwen_d", dict(synth.CANONS["qwen2.5-0.5b"], layers=2, max_len=1024, name="qwen0.5b-2l"), 22,
     dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=8)),
]
QWEN_FILL = 776          # KV positions filled with seeded values before each case
# (rows, first position): 1-row decode passes and 5-row verify passes; 511..515
# and 636..640 cross a 16-position page boundary, 763..767 ends at the fill
QWEN_CASES = [(1, 511), (1, 640), (1, 767), (5, 511), (5, 636), (5, 763)]
QWEN_LOGIT_SAMPLE = 2048


def qwen_kv_fill(canon, seed, layer):
    """Seeded fp16 K and V (QWEN_FILL, kv_heads, head_dim) for one layer."""
    rng = np.random.default_rng([int(seed), 1000 + int(layer)])
    shape = (QWEN_FILL, canon["kv_heads"], canon["head_dim"])
    k = (rng.standard_normal(shape, dtype=np.float32) * np.float32(1.5)).astype(np.float16)
    v = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    return k, v


def qwen_case_tokens(canon, seed, case):
    """Token ids of one case's rows (the first `rows` of these)."""
    return np.random.default_rng([int(seed), 2000 + int(case)]).integers(0, canon["vocab"], 8).tolist()


def qwen_logit_index(vocab):
    """The logit entries the fixture stores for every row."""
    return np.sort(np.random.default_rng(77).choice(vocab, QWEN_LOGIT_SAMPLE, replace=False))
