"""Shared helpers of the GPU tests (not a test module)."""
import numpy as np


def random_codes(rng, out, k, bits, block, zero_blocks=0):
    """Random shard-format codes and fp16 scales for an (out, k) weight."""
    nb = k // block
    if bits == 4:
        q = rng.integers(-8, 8, size=(out, k), dtype=np.int32)
        from oracle.quant import pack_int4
        packed = pack_int4(q)
    else:
        q = rng.integers(-128, 128, size=(out, k), dtype=np.int32)
        packed = q.astype(np.int8)
    scale = (np.abs(rng.standard_normal((out, nb))) * 0.003 + 1e-4).astype(np.float16)
    for _ in range(zero_blocks):
        scale[rng.integers(out), rng.integers(nb)] = 0
    return packed, scale


def rel_err(got, ref):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    return float(np.max(np.abs(got - ref)) / max(1e-6, float(np.max(np.abs(ref)))))


def ulp_diff(got, ref):
    """Per-element distance in fp16 units in the last place."""
    a = np.asarray(got, np.float16).view(np.int16).astype(np.int32)
    b = np.asarray(ref, np.float16).view(np.int16).astype(np.int32)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return np.abs(a - b)


def ref_matmul(x, w):
    """fp32-accumulated x . w^T rounded once to fp16 (numpy's half matmul)."""
    return (np.asarray(x, np.float32) @ np.asarray(w, np.float32).T).astype(np.float16)


def prefill(model, kv, tokens, pos0=0, chunk=16):
    """Run the model over tokens at positions pos0.. (no head), in chunks."""
    for i in range(0, len(tokens), chunk):
        model.forward(kv, tokens[i:i + chunk], pos0 + i, logits=False, argmax=False)


def greedy_plain(model, kv, prompt, n_new):
    """The reference's plain greedy loop (androidllm/engine.py:347-399) on the device."""
    prefill(model, kv, prompt[:-1])
    tok, pos, out = prompt[-1], len(prompt) - 1, []
    for _ in range(n_new):
        _, am = model.forward(kv, [tok], pos)
        tok = int(am[0])
        pos += 1
        out.append(tok)
    return out


def greedy_spec(target, draft, tkv, dkv, prompt, n_new, k):
    """Speculative greedy generate (androidllm/engine.py:347-387) via SpecDecoder;
    returns (tokens, steps, accepted, bonus)."""
    from androidllm_b200.ops import SpecDecoder
    prefill(target, tkv, prompt[:-1])
    prefill(draft, dkv, prompt)
    s = SpecDecoder(target, draft, tkv, dkv, k)
    s.begin(prompt[-1], len(prompt) - 1)
    out, steps, acc, bonus = [], 0, 0, 0
    while len(out) < n_new:
        emitted, n_acc = s.run(1)
        steps += 1
        for i, t in enumerate(emitted):
            if len(out) >= n_new:
                break
            out.append(t)
            if i < n_acc[0]:
                acc += 1
            else:
                bonus += 1
    s.close()
    return out, steps, acc, bonus
