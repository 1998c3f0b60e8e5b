"""The GGUF parity cases behind gguf.npz, shared by the script that generates
the fixture from the reference's GGUF reader (make_gguf_golden.py) and the
tests.

* Block cases: for every GGML type the reference reads, a (6, 64) tensor of
  seeded random block bytes (fp16 scales and offsets drawn from a sane range,
  one all-zero block).  The fixture holds the bytes and the reference
  reader's fp32 values.
* Two small models written as GGUF files by this package's writer with 32-bit
  tensor dimensions (the form the reference reads):
  - gguf_a: the reference GGUF test's shape (hidden 64, 2 layers, 4/2 heads,
    FFN 96, vocab 64), Q4_0 attention, Q8_0 MLP, Q8_0 embedding, F32 norms,
    tied head;
  - gguf_b: hidden 128, 2 layers, 4/2 heads of 32, FFN 352 (not a multiple
    of 64), vocab 256, Q4_0 projections but Q8_0 down, F16 embedding, BF16
    norms, untied Q4_0 head.
  The fixture holds the sha256 of each file and of the reference reader's
  fp32 decode of each tensor.
"""
import numpy as np

from androidllm_b200 import gguf

BLOCK_SHAPE = (6, 64)
BLOCK_TYPES = ["F32", "F16", "BF16", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q8_1"]
_BY_NAME = {v: k for k, v in gguf.TYPE_NAMES.items()}


def block_bytes(type_name, seed=0):
    """Seeded raw bytes of a BLOCK_SHAPE tensor of one GGML type."""
    gtype = _BY_NAME[type_name]
    rng = np.random.default_rng([seed, gtype])
    n = BLOCK_SHAPE[0] * BLOCK_SHAPE[1]
    if type_name == "F32":
        return rng.standard_normal(n).astype(np.float32).tobytes()
    if type_name == "F16":
        return rng.standard_normal(n).astype(np.float16).tobytes()
    if type_name == "BF16":
        return (rng.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    size = gguf.tensor_bytes(gtype, (n,))
    nb = n // 32
    buf = rng.integers(0, 256, size, dtype=np.uint8).reshape(nb, -1)
    d = (rng.uniform(0.001, 0.05, nb) * rng.choice([-1.0, 1.0], nb)).astype(np.float16)
    buf[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    if type_name in ("Q4_1", "Q5_1", "Q8_1"):
        m = rng.uniform(-0.1, 0.1, nb).astype(np.float16)
        buf[:, 2:4] = m.view(np.uint8).reshape(nb, 2)
    buf[3] = 0                       # an all-zero block (d = 0)
    return buf.tobytes()


def _meta(arch, canon):
    return {"general.architecture": arch, "general.name": canon["name"],
            f"{arch}.block_count": canon["layers"], f"{arch}.embedding_length": canon["hidden"],
            f"{arch}.feed_forward_length": canon["intermediate"],
            f"{arch}.attention.head_count": canon["heads"], f"{arch}.attention.head_count_kv": canon["kv_heads"],
            f"{arch}.attention.max_position_embeddings": canon["max_len"],
            f"{arch}.rope.freq_base": canon["rope_theta"],
            f"{arch}.attention.layer_norm_rms_epsilon": canon["rms_eps"], f"{arch}.vocab_size": canon["vocab"],
            "tokenizer.ggml.model": "gpt2"}


GGUF_A = dict(model_type="qwen2", hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, intermediate=96,
              vocab=64, rope_theta=10000.0, rms_eps=1e-6, max_len=128, tied=True, name="gguf-a")
GGUF_B = dict(model_type="qwen2", hidden=128, layers=2, heads=4, kv_heads=2, head_dim=32, intermediate=352,
              vocab=256, rope_theta=1e6, rms_eps=1e-6, max_len=256, tied=False, name="gguf-b")
GGUF_MODELS = {"gguf_a": (GGUF_A, 31), "gguf_b": (GGUF_B, 32)}
GGUF_PROMPT = [3, 17, 9, 41, 5, 28, 60, 12, 33]


def _bf16_raw(x):
    x = np.asarray(x, np.float32)
    return gguf.RawTensor(gguf.T_BF16, (x.view(np.uint32) >> 16).astype(np.uint16).tobytes(), x.shape)


def model_tensors(name):
    """{gguf tensor name: RawTensor | (type, array)} of one case model."""
    canon, seed = GGUF_MODELS[name]
    rng = np.random.default_rng(seed)
    h, f, v = canon["hidden"], canon["intermediate"], canon["vocab"]
    kvd = canon["kv_heads"] * canon["head_dim"]
    b = name == "gguf_b"
    t = {}

    def w(o, i, std=0.05):
        return (rng.standard_normal((o, i)) * std).astype(np.float32)

    def norm():
        x = (1.0 + 0.1 * rng.standard_normal(h)).astype(np.float32)
        return _bf16_raw(x) if b else (gguf.T_F32, x)
    if b:
        t["token_embd.weight"] = (gguf.T_F16, (rng.standard_normal((v, h)) * 0.5).astype(np.float16))
    else:
        t["token_embd.weight"] = (gguf.T_Q8_0, w(v, h, 0.5))
    t["output_norm.weight"] = norm()
    if b:
        t["output.weight"] = (gguf.T_Q4_0, w(v, h, 0.2))
    for i in range(canon["layers"]):
        p = f"blk.{i}."
        t[p + "attn_norm.weight"] = norm()
        t[p + "ffn_norm.weight"] = norm()
        for proj, o, n in (("attn_q", h, h), ("attn_k", kvd, h), ("attn_v", kvd, h), ("attn_output", h, h),
                           ("ffn_gate", f, h), ("ffn_up", f, h), ("ffn_down", h, f)):
            mlp = proj.startswith("ffn")
            gt = (gguf.T_Q8_0 if proj == "ffn_down" else gguf.T_Q4_0) if b else (gguf.T_Q8_0 if mlp else gguf.T_Q4_0)
            t[p + proj + ".weight"] = (gt, w(o, n))
    return t


def write_model(name, path, order="reference", dims64=False):
    canon, _ = GGUF_MODELS[name]
    gguf.write_gguf(path, _meta("qwen2", canon), model_tensors(name), dims64=dims64, order=order)
