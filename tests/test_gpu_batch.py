"""Batched sessions (androidllm/batching.py:32-272; the reference steps one
session per visit): multi-sequence passes over a multi-slot paged KV equal
each sequence's own forward bit for bit, and batched generation equals
generate() per prompt, greedy and sampling, through run_batch, the
BatchScheduler thread and SessionPool prefix reuse."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


@pytest.mark.parametrize("name", ["toyu", "minq"])
def test_forward_seqs_equals_single_sequence_forwards(ctx, model_dirs, name):
    """Three sequences in the slots of one cache (prompts of 40, 7 and 200
    tokens, prefilled into slots 2, 0 and 3), then one pass of 1 + 5 + 3 rows:
    logits, argmax and the new KV entries equal three single-sequence
    forwards on separate caches, bit for bit."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs[name])
    rng = np.random.default_rng(12)
    V = m.canon["vocab"]
    lens = [40, 7, min(200, int(m.canon["max_len"]) - 24)]
    slots = [2, 0, 3]
    prompts = [rng.integers(0, V, n).tolist() for n in lens]
    rows = [1, 5, 3]
    new = [rng.integers(0, V, r).tolist() for r in rows]
    cap = max(lens) + 16
    multi = DeviceKV(m, cap, 16, slots=4)
    singles = [DeviceKV(m, cap, 16) for _ in prompts]
    for p, s, kv in zip(prompts, slots, singles):
        m.prefill(multi, p, 0, slot=s)
        m.prefill(kv, p, 0)
    lg_m, am_m = m.forward_seqs(multi, [(s, t, len(p)) for s, t, p in zip(slots, new, prompts)], logits=True)
    for i, (p, t, kv) in enumerate(zip(prompts, new, singles)):
        lg, am = m.forward(kv, t, len(p), logits=True)
        assert np.array_equal(lg_m[i].view(np.uint32), lg.view(np.uint32)), i
        assert np.array_equal(am_m[i], am), i
        for li in range(m.canon["layers"]):
            k1, v1 = multi.read(li, 0, len(p) + len(t), slot=slots[i])
            k2, v2 = kv.read(li, 0, len(p) + len(t))
            assert np.array_equal(k1.view(np.uint16), k2.view(np.uint16)), (i, li)
            assert np.array_equal(v1.view(np.uint16), v2.view(np.uint16)), (i, li)


@pytest.mark.parametrize("name", ["toyu", "minq"])
def test_pass_of_64_rows_equals_single_sequence_forwards(ctx, model_dirs, name):
    """A pass of 64 rows (13 sequences of 1-8 rows: four 16-row groups of
    the GEMV, groups cutting through sequences) equals each sequence's own
    forward bit for bit: logits, argmax and the new KV entries; sampling
    rows past the 16th of the pass matches sampling them alone."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs[name])
    assert m.max_pass_rows() == 64
    rng = np.random.default_rng(31)
    V = m.canon["vocab"]
    rows = [5, 5, 1, 8, 5, 3, 7, 5, 2, 6, 5, 4, 8]
    assert sum(rows) == 64
    lens = [int(rng.integers(3, 90)) for _ in rows]
    slots = list(range(len(rows)))[::-1]
    prompts = [rng.integers(0, V, n).tolist() for n in lens]
    new = [rng.integers(0, V, r).tolist() for r in rows]
    cap = 112
    multi = DeviceKV(m, cap, 16, slots=len(rows))
    for p, s in zip(prompts, slots):
        m.prefill(multi, p, 0, slot=s)
    lg_m, am_m = m.forward_seqs(multi, [(s, t, len(p)) for s, t, p in zip(slots, new, prompts)], logits=True)
    u = rng.random(64)
    picks_m = m.sample_rows(0, 64, 0.8, 0.9, 0.0, u)
    for i, (p, t) in enumerate(zip(prompts, new)):
        kv = DeviceKV(m, cap, 16)
        m.prefill(kv, p, 0)
        lg, am = m.forward(kv, t, len(p), logits=True)
        assert np.array_equal(lg_m[i].view(np.uint32), lg.view(np.uint32)), i
        assert np.array_equal(am_m[i], am), i
        r0 = sum(rows[:i])
        assert np.array_equal(picks_m[r0:r0 + rows[i]], m.sample_rows(0, rows[i], 0.8, 0.9, 0.0, u[r0:r0 + rows[i]])), i
        for li in range(m.canon["layers"]):
            k1, v1 = multi.read(li, 0, len(p) + len(t), slot=slots[i])
            k2, v2 = kv.read(li, 0, len(p) + len(t))
            assert np.array_equal(k1.view(np.uint16), k2.view(np.uint16)), (i, li)
            assert np.array_equal(v1.view(np.uint16), v2.view(np.uint16)), (i, li)
    with pytest.raises(Exception):
        m.forward_seqs(multi, [(s, [1] * 5, 90) for s in range(13)])   # 65 rows


def test_pass_of_40_rows_at_the_targets_layer_shapes(ctx, tmp_path):
    """Eight sessions' verify rows (5 each) in one pass on 2 layers of the
    benchmark target's shapes (hidden 1536, 12/2 heads of 128, FFN 8960,
    int4 attention / int8 MLP, tied int8 head of 4096 rows): 32-row GEMV
    groups, split K across CTAs (the 8960-column down projection), equal to
    each sequence's own 5-row forward bit for bit."""
    from androidllm_b200 import shard, synth
    from androidllm_b200.ops import DeviceKV, DeviceModel
    canon = dict(synth.CANONS["qwen2.5-1.5b"], layers=2, vocab=4096, max_len=512, name="qwen1.5b-2l-v4096")
    d = str(tmp_path / "q")
    shard.shard_from_tensors(synth.synth_tensors(canon, seed=8), canon, d, attn_bits=4, mlp_bits=8, block=64,
                             embed_bits=8)
    m = DeviceModel.from_dir(ctx, d)
    rng = np.random.default_rng(40)
    lens = [int(rng.integers(20, 200)) for _ in range(8)]
    prompts = [rng.integers(0, 4096, n).tolist() for n in lens]
    new = [rng.integers(0, 4096, 5).tolist() for _ in lens]
    multi = DeviceKV(m, 224, 16, slots=8)
    for s, p in enumerate(prompts):
        m.prefill(multi, p, 0, slot=s)
    lg_m, am_m = m.forward_seqs(multi, [(s, t, len(p)) for s, (t, p) in enumerate(zip(new, prompts))], logits=True)
    for i, (p, t) in enumerate(zip(prompts, new)):
        kv = DeviceKV(m, 224, 16)
        m.prefill(kv, p, 0)
        lg, am = m.forward(kv, t, len(p), logits=True)
        assert np.array_equal(lg_m[i].view(np.uint32), lg.view(np.uint32)), i
        assert np.array_equal(am_m[i], am), i
        for li in range(2):
            k1, v1 = multi.read(li, 0, len(p) + 5, slot=i)
            k2, v2 = kv.read(li, 0, len(p) + 5)
            assert np.array_equal(k1.view(np.uint16), k2.view(np.uint16)), (i, li)
            assert np.array_equal(v1.view(np.uint16), v2.view(np.uint16)), (i, li)


def test_slot_pages_remapped(ctx, model_dirs):
    """A slot whose pages are remapped (alm_kv_set_pages) still gives the
    single-sequence forward's logits."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs["toyu"])
    rng = np.random.default_rng(5)
    p = rng.integers(0, m.canon["vocab"], 60).tolist()
    multi = DeviceKV(m, 96, 16, slots=3)         # 6 pages of 16 positions per slot, 18 in all
    multi.set_pages(1, [17, 3, 12, 0, 9, 16])   # slot 1 on pages of all three slots
    m.prefill(multi, p, 0, slot=1)
    single = DeviceKV(m, 96, 16)
    m.prefill(single, p, 0)
    lg_m, _ = m.forward_seqs(multi, [(1, [7], 60)], logits=True)
    lg, _ = m.forward(single, [7], 60, logits=True)
    assert np.array_equal(lg_m[0].view(np.uint32), lg.view(np.uint32))


def _prompts(n, vocab, seed=3):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, int(rng.integers(12, 180))).tolist() for _ in range(n)]


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_generate_batch_equals_generate(model_dirs, temperature):
    """Five sessions advanced together (spec k = 4) give every prompt the
    tokens generate() gives it alone (sampling: the same seed)."""
    from androidllm_b200.engine import LayerStreamingEngine
    eng = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    prompts = _prompts(5, 32000)
    seeds = [101, 102, 103, 104, 105]
    got = eng.generate_batch(prompts, max_new_tokens=40, temperature=temperature, top_p=0.9, seeds=seeds)
    for p, s, g in zip(prompts, seeds, got):
        ref = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4, seed=s,
                                   _ctx=eng.ctx)
        want = ref.generate(p, max_new_tokens=40, temperature=temperature, top_p=0.9)
        assert g == want
        ref.close()
    assert eng.batch_runner().free_slots() == eng.batch_runner().slots
    eng.close()


def test_continuous_batching_queue(model_dirs):
    """Five prompts with at most two sessions active (a finished session's
    slot takes the next prompt): the tokens of each prompt are unchanged."""
    from androidllm_b200.engine import LayerStreamingEngine
    eng = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    prompts = _prompts(5, 32000, seed=21)
    outs = [8, 30, 12, 25, 5]
    all_at_once = eng.generate_batch(prompts, max_new_tokens=outs, temperature=0.0)
    two = eng.generate_batch(prompts, max_new_tokens=outs, temperature=0.0, max_active=2)
    assert two == all_at_once
    assert [len(g) for g in two] == outs
    eng.close()


def test_generate_batch_without_draft(model_dirs):
    """Sessions of an engine without a draft take plain batched steps (one
    row per session per pass): equal to generate() per prompt."""
    from androidllm_b200.engine import LayerStreamingEngine
    eng = LayerStreamingEngine(model_dirs["toyu"])
    prompts = _prompts(6, 32000, seed=4)
    seeds = list(range(6))
    got = eng.generate_batch(prompts, max_new_tokens=20, temperature=0.8, top_p=0.9, seeds=seeds)
    for p, s, g in zip(prompts, seeds, got):
        ref = LayerStreamingEngine(model_dirs["toyu"], seed=s, _ctx=eng.ctx)
        assert g == ref.generate(p, max_new_tokens=20, temperature=0.8, top_p=0.9)
        ref.close()
    eng.close()


def test_scheduler_and_pool(model_dirs):
    """BatchScheduler: four sessions submitted together finish with
    generate()'s tokens; the done callback puts them in a SessionPool, and
    a follow-up prompt sharing a prefix reuses a slot and still matches."""
    from androidllm_b200.batching import BatchScheduler, Session, SessionPool
    from androidllm_b200.engine import LayerStreamingEngine
    eng = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    ref = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4, _ctx=eng.ctx)
    pool = SessionPool(eng, max_pooled=4)
    sched = BatchScheduler(eng, max_slots=4)
    prompts = _prompts(4, 32000, seed=9)
    done = threading.Event()
    finished = []

    def cb(sess):
        finished.append(sess)
        pool.put(sess)
        if len(finished) == len(prompts):
            done.set()

    sessions = [Session(eng, p, max_new_tokens=24, temperature=0.0) for p in prompts]
    assert all(sched.submit(s, cb) for s in sessions)
    assert not sched.submit(Session(eng, prompts[0], max_new_tokens=4, temperature=0.0), cb)   # slots full
    assert done.wait(120)
    for s, p in zip(sessions, prompts):
        assert s.error is None
        assert s.generated == ref.generate(p, max_new_tokens=24, temperature=0.0)
    snap = sched.snapshot()
    assert set(snap) == {"active", "queued", "max", "completed", "rejected"}
    assert snap["completed"] == 4 and snap["rejected"] == 1
    # prefix reuse through the pool: the first prompt plus its answer plus new tokens
    follow = prompts[0] + sessions[0].generated[:10] + [5, 6, 7]
    s2, pfx = pool.acquire(follow)
    assert pfx > len(prompts[0]) and s2.slot == sessions[0].slot
    s2.max_new_tokens = 16
    s2.temperature = 0.0
    done2 = threading.Event()
    assert sched.submit(s2, lambda s: done2.set())
    assert done2.wait(60)
    # the same KV history through generate()'s own prefix reuse
    ref.generate(prompts[0], max_new_tokens=24, temperature=0.0)
    assert s2.generated == ref.generate(follow, max_new_tokens=16, temperature=0.0)
    sched.close()
    ref.close()
    eng.close()
