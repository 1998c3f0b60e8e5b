"""The Python drop-in API on the GPU, driven the way the reference's own tests
drive the reference (androidllm tests/test_streaming.py:119-151 and
tests/test_spec.py:47-100).

* ``LlamaModel(canon, embed, final_norm, lm_head)`` fed the reference's dicts
  of dequantized fp16 matrices, with ``prepare_kv(max_len)`` and
  ``layer_forward(x, layer, kv[li], pos)`` per layer and position, then
  ``logits`` — against the oracle run the same way, at the 1e-2 tolerance.
* ``LayerStreamingEngine.generate(temperature=0)`` with a 2-layer draft and
  ``spec_k=4`` — the reference's own token stream and speculative statistics.
"""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import rel_err, ulp_diff

from oracle import io as oio
from oracle import llama as ollama

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _run_like_test_streaming(model, layers, prompt, max_len):
    """tests/test_streaming.py:119-126: x = embed[prompt[0]], then every
    position through every layer, feeding each output back in."""
    kv = model.prepare_kv(max_len)
    x = model.embed[prompt[0]].reshape(1, -1)
    per_pos = []
    for pos in range(len(prompt)):
        for li in range(len(layers)):
            x = model.layer_forward(x, layers[li], kv[li], pos)
        per_pos.append(np.asarray(x, np.float16).copy())
    return per_pos, model.logits(x)


@pytest.mark.parametrize("name", ["tiny", "minq", "toy"])
def test_llama_model_dropin_with_fp16_dicts(model_dirs, name):
    from androidllm_b200.models.llama import LlamaModel
    canon, embed, fnorm, head, layers = oio.load_model(model_dirs[name])
    prompt = [3, 7, 11, 5, 1, 0, 9]
    dev = LlamaModel(canon, embed, fnorm, head)
    ref = ollama.OracleModel(canon, embed, fnorm, head)
    got_states, got_lg = _run_like_test_streaming(dev, layers, prompt, 64)
    ref_states, ref_lg = _run_like_test_streaming(ref, layers, prompt, 64)
    for pos, (a, b) in enumerate(zip(got_states, ref_states)):
        assert rel_err(a, b) < TOL, (name, pos)
    assert got_lg.shape == ref_lg.shape == (1, canon["vocab"])
    assert got_lg.dtype == np.float32
    assert rel_err(got_lg, ref_lg) < TOL
    print(f"{name}: logits bit-identical {np.mean(ulp_diff(got_lg, ref_lg) == 0):.3f}")
    # the KV view returns the reference cache layout
    k, v = dev.prepare_kv(8)[0].read(0, 2)
    assert k.shape == v.shape == (2, canon["kv_heads"], canon["head_dim"]) and k.dtype == np.float16


def test_llama_model_dropin_with_shard_projections(model_dirs):
    """The same model fed shard-format projections (QuantProj, no host
    dequantization) gives the same results as the fp16 dicts within 1e-2."""
    from androidllm_b200.models.llama import LlamaModel
    from androidllm_b200.ops import load_manifest, read_layer
    d = model_dirs["minq"]
    canon, embed, fnorm, head, layers = oio.load_model(d)
    man = load_manifest(d)
    qlayers = [read_layer(d, man, i) for i in range(canon["layers"])]
    prompt = [5, 17, 900, 3, 44]
    a = _run_like_test_streaming(LlamaModel(canon, embed, fnorm, head), qlayers, prompt, 32)
    b = _run_like_test_streaming(ollama.OracleModel(canon, embed, fnorm, head), layers, prompt, 32)
    assert rel_err(a[1], b[1]) < TOL
    for x, y in zip(a[0], b[0]):
        assert rel_err(x, y) < TOL


def test_engine_generate_greedy_spec_equals_reference(model_dirs):
    """LayerStreamingEngine.generate(temperature=0) with the 2-layer prefix
    draft and spec_k=4 (the public path the benchmark's e2e times): the
    reference's 128-token speculative stream and its step / draft / accepted
    / bonus counts (tests/golden/toy.npz, written by the reference)."""
    from androidllm_b200.engine import LayerStreamingEngine
    g = golden("toy.npz")
    eng = LayerStreamingEngine(model_dirs["toy"], draft_dir=model_dirs["toy_draft"], spec_k=4)
    prompt = [int(t) for t in g["prompt"]]
    out = eng.generate(prompt, max_new_tokens=128, temperature=0.0, top_p=1.0)
    assert out == g["spec"].tolist()
    sp = eng.snapshot()["spec"]
    assert [sp["steps"], sp["draft_tokens"], sp["accepted"], sp["bonus"]] == g["spec_stats"].tolist()
    # plain greedy through the same engine: the reference's plain stream
    plain = LayerStreamingEngine(model_dirs["toy"]).generate(prompt, max_new_tokens=128, temperature=0.0)
    assert plain == g["plain"].tolist()
    eng.close()
