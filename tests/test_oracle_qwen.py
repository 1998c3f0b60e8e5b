"""CPU pin of the oracle at the benchmark's layer shapes against the
reference's own outputs (tests/golden/qwen.npz, written by running the
reference): this repository's shard writer produces the reference writer's
bytes for the 2-layer Qwen2.5-1.5B / 0.5B-shaped models, and the oracle's
layer states and logits equal the reference's bit for bit."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest
from conftest import GOLDEN, golden

sys.path.insert(0, GOLDEN)
from qwen_cases import QWEN_CASES, QWEN_FILL, QWEN_MODELS, qwen_case_tokens, qwen_kv_fill  # noqa: E402

pytestmark = pytest.mark.slow


@pytest.fixture(scope="module")
def written(tmp_path_factory):
    from androidllm_b200 import shard, synth
    root = tmp_path_factory.mktemp("qwen_cpu")
    out = {}
    for name, canon, seed, kw in QWEN_MODELS:
        d = str(root / name)
        shard.shard_from_tensors(synth.synth_tensors(canon, seed=seed), canon, d, **kw)
        out[name] = d
    return out


@pytest.mark.parametrize("name", ["qwen_t", "qwen_d"])
def test_writer_bytes_equal_reference_at_benchmark_shapes(written, name):
    g = golden("qwen.npz")
    ref = json.loads(str(g[f"{name}_files"]))
    d = written[name]
    got = {}
    for fn in sorted(os.listdir(d)):
        with open(os.path.join(d, fn), "rb") as f:
            got[fn] = hashlib.sha256(f.read()).hexdigest()
    assert got == ref


@pytest.mark.parametrize("name,ci", [("qwen_t", 3), ("qwen_d", 2)])
def test_oracle_equals_reference_at_benchmark_shapes(written, name, ci):
    from oracle import io as oio
    from oracle import llama as ollama
    g = golden("qwen.npz")
    canon, embed, fnorm, head, layers = oio.load_model(written[name])
    seed = {n: s for n, _, s, _ in QWEN_MODELS}[name]
    om = ollama.OracleModel(canon, embed, fnorm, head)
    kv = om.prepare_kv(QWEN_FILL + 8)
    for li in range(canon["layers"]):
        k, v = qwen_kv_fill(canon, seed, li)
        kv[li][0][:QWEN_FILL] = k
        kv[li][1][:QWEN_FILL] = v
    rows, pos0 = QWEN_CASES[ci]
    row0 = sum(r for r, _ in QWEN_CASES[:ci])
    for r, tok in enumerate(qwen_case_tokens(canon, seed, ci)[:rows]):
        x = embed[tok].reshape(1, -1)
        for li in range(canon["layers"]):
            x = om.layer_forward(x, layers[li], kv[li], pos0 + r)
            assert np.array_equal(x[0].view(np.uint16), g[f"{name}_states"][ci][r, li].view(np.uint16)), (r, li)
        lg = om.logits(x).reshape(-1).astype(np.float16)
        assert hashlib.sha256(lg.tobytes()).hexdigest() == str(g[f"{name}_hash"][row0 + r])
        assert int(np.argmax(lg)) == int(g[f"{name}_argmax"][row0 + r])
