"""GGUF models loaded straight to the device (Q4_0 / Q8_0 blocks kept as int4
/ int8 with 32-column blocks): the device's dequantized weights equal the
fp16 rounding of the reference reader's values, and the forward's logits and
greedy tokens match the oracle model on those weights."""
import sys

import numpy as np
import pytest
from conftest import GOLDEN
from gpu_helpers import rel_err

sys.path.insert(0, GOLDEN)
from gguf_cases import GGUF_MODELS, GGUF_PROMPT, write_model  # noqa: E402

from oracle import llama as ollama  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


def _oracle(gf):
    canon = gf.canon()
    layers = []
    for i in range(canon["layers"]):
        layer = {}
        for gname, base in (("attn_q", "q"), ("attn_k", "k"), ("attn_v", "v"), ("attn_output", "o"),
                            ("ffn_gate", "gate"), ("ffn_up", "up"), ("ffn_down", "down")):
            layer[base] = gf.fp16(f"blk.{i}.{gname}.weight")
        layer["n_in"] = gf.fp16(f"blk.{i}.attn_norm.weight").reshape(-1)
        layer["n_post"] = gf.fp16(f"blk.{i}.ffn_norm.weight").reshape(-1)
        layers.append(layer)
    head = gf.fp16("output.weight") if "output.weight" in gf.tensors else None
    return ollama.OracleModel(canon, gf.fp16("token_embd.weight"), gf.fp16("output_norm.weight").reshape(-1),
                              head), layers


@pytest.mark.parametrize("name", sorted(GGUF_MODELS))
def test_gguf_model_matches_oracle(ctx, tmp_path, name):
    from androidllm_b200.gguf import T_Q4_0, T_Q8_0, GGUFFile, device_model_from_gguf
    from androidllm_b200.ops import DeviceKV, QWeight
    path = str(tmp_path / f"{name}.gguf")
    write_model(name, path)
    gf = GGUFFile(path)
    # device dequantization of every direct projection
    for tname, t in gf.tensors.items():
        if t["type"] in (T_Q4_0, T_Q8_0) and tname != "token_embd.weight":
            w = QWeight(ctx, gf.projection(tname))
            assert np.array_equal(w.dequant().view(np.uint16), gf.fp16(tname).view(np.uint16)), tname
            w.free()
    m = device_model_from_gguf(ctx, path)
    om, layers = _oracle(gf)
    n_new = 12
    kv = DeviceKV(m, len(GGUF_PROMPT) + n_new + 4)
    okv = om.prepare_kv(len(GGUF_PROMPT) + n_new + 4)
    toks, otoks = list(GGUF_PROMPT), list(GGUF_PROMPT)
    for pos in range(len(GGUF_PROMPT) + n_new - 1):
        lg, am = m.forward(kv, [toks[pos]], pos, logits=True)
        x = om.forward(layers, otoks[pos], okv, pos)
        olg = om.logits(x)[0]
        assert rel_err(lg[0], olg) < 1e-2, pos
        if pos >= len(GGUF_PROMPT) - 1:
            srt = np.sort(olg)
            if int(am[0]) != int(np.argmax(olg)):
                # only a near-tie of the oracle's logits may flip the greedy pick
                assert srt[-1] - srt[-2] <= 2 * float(np.spacing(np.float16(abs(srt[-1])))), pos
                break
            toks.append(int(am[0]))
            otoks.append(int(am[0]))
    print(f"{name}: {len(toks) - len(GGUF_PROMPT)} greedy tokens equal to the oracle's")
