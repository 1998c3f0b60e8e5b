"""The opt-in one-launch attention (csrc/attn_fused.cu) against the two passes
it replaces: the same probabilities, P.V sums in another fp32 order, so
logits agree to fp16 rounding; verify rows equal single-row passes bit for
bit with it too; and it matches the reference's states on a golden model."""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import prefill, rel_err

pytestmark = pytest.mark.gpu


def _run(fused, model_dir, toks):
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    c = Context(0)
    c.set_attn_fused(fused)
    m = DeviceModel.from_dir(c, model_dir)
    kv = DeviceKV(m, 256, 16)
    prefill(m, kv, toks[:100])
    lg5, _ = m.forward(kv, toks[100:105], 100, logits=True)
    kv1 = DeviceKV(m, 256, 16)
    prefill(m, kv1, toks[:100])
    lg1 = [m.forward(kv1, [t], 100 + i, logits=True)[0][0] for i, t in enumerate(toks[100:105])]
    return lg5, np.stack(lg1)


@pytest.mark.parametrize("name", ["toyu", "minq"])
def test_fused_attention_matches_two_passes(model_dirs, name):
    toks = np.random.default_rng(2).integers(0, 1000, 110).tolist()
    f5, f1 = _run(True, model_dirs[name], toks)
    t5, t1 = _run(False, model_dirs[name], toks)
    # verify rows == single rows, bit for bit, under each kernel
    assert np.array_equal(f5.view(np.uint32), f1.view(np.uint32))
    assert np.array_equal(t5.view(np.uint32), t1.view(np.uint32))
    assert rel_err(f5, t5) < 1e-2
    exact = float(np.mean(f5.view(np.uint32) == t5.view(np.uint32)))
    print(f"{name}: {exact:.3f} of the logits bit-identical between the one-launch and the two-pass attention")


def test_fused_attention_against_reference_states(model_dirs):
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    from oracle import io as oio
    g = golden("toyu.npz")
    c = Context(0)
    c.set_attn_fused(True)
    m = DeviceModel.from_dir(c, model_dirs["toyu"])
    emb = oio.load_model(model_dirs["toyu"])[1]
    kv = DeviceKV(m, 512, 16)
    prompt = [int(t) for t in g["prompt"]]
    n_pos = g["states"].shape[0]
    for pos, tok in enumerate(prompt[:n_pos]):
        x = emb[tok].reshape(1, -1)
        for li in range(m.canon["layers"]):
            x = m.layer_forward(li, kv, x, pos)
            assert rel_err(x, g["states"][pos, li].reshape(1, -1)) < 1e-2, (pos, li)
