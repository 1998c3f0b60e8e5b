"""Host logic of batched sessions (androidllm_b200/batching.py) without a GPU:
a session's bookkeeping of emitted tokens (stop ids, budget, the cached
token list), its uniform stream (consumed in the reference's per-step count),
the pool's prefix matching and the per-session KV size of the reference's
budget rule (androidllm/batching.py:22-28)."""
import numpy as np
import pytest

from androidllm_b200 import batching


class _Runner:
    slots = 8

    def __init__(self):
        self.released = []

    def release_slot(self, slot):
        self.released.append(slot)


class _Engine:
    def __init__(self, spec_k=4, draft=True):
        self.ctx_len = 64
        self.canon = {"layers": 4, "kv_heads": 2, "head_dim": 32}
        self.spec_k = spec_k
        self.draft = object() if draft else None
        self.stats = {"tokens_served": 0}
        self._runner = _Runner()

    def batch_runner(self):
        return self._runner


def test_kv_bytes_per_session():
    e = _Engine()
    assert batching.kv_bytes_per_session(e) == 64 * 2 * 32 * 2 * 2 * 4
    assert batching.kv_bytes_per_session(e, 10) == 10 * 2 * 32 * 2 * 2 * 4


def test_advance_counts_stops_and_budget():
    e = _Engine()
    s = batching.Session(e, [1, 2, 3], max_new_tokens=5, temperature=0.0, stop_ids=(99,))
    s.pos, s.token, s.prefilled = 2, 3, True
    s._kv_ids = [1, 2]
    s._advance([7, 8, 9], 2)            # two candidates accepted, a bonus
    assert s.generated == [7, 8, 9] and s.pos == 5 and s.token == 9 and not s.done
    assert s._kv_ids == [1, 2, 3, 7, 8]
    assert e.stats["spec_accepted"] == 2 and e.stats["spec_bonus"] == 1 and e.stats["tokens_served"] == 3
    s._advance([10, 99, 11], 1)          # a stop id ends the session and is not emitted
    assert s.generated == [7, 8, 9, 10] and s.done and s.token == 99
    t = batching.Session(e, [1, 2], max_new_tokens=2, temperature=0.0)
    t.pos, t.token, t.prefilled = 1, 2, True
    t._advance([4, 5, 6], 2)             # budget of 2: the rest is dropped
    assert t.generated == [4, 5] and t.done


def test_uniform_stream_consumption():
    """k draft draws, then one per verified row up to the first rejection and
    the bonus: the next step starts after K + accepted + 1 draws."""
    e = _Engine(spec_k=4)
    s = batching.Session(e, [1, 2], temperature=0.8, seed=7)
    ref = np.random.default_rng(7).random(10000)
    s._ensure_draws(9)
    assert np.array_equal(s._draws(9), ref[:9])
    s._consume(4 + 2 + 1)
    s._ensure_draws(9)
    assert np.array_equal(s._draws(9), ref[7:16])
    g = batching.Session(e, [1, 2], temperature=0.0)
    g._ensure_draws(9)
    assert g._draws(9) is None
    g._consume(9)
    assert g._u_used == 0


def test_pool_prefix_match_and_eviction():
    e = _Engine()
    pool = batching.SessionPool(e, max_pooled=2)
    a = batching.Session(e, [1, 2, 3, 4], temperature=0.0)
    a.slot, a._kv_ids = 3, [1, 2, 3, 4, 5, 6]
    b = batching.Session(e, [9, 9], temperature=0.0)
    b.slot, b._kv_ids = 4, [9, 9]
    pool.put(a)
    pool.put(b)
    assert len(pool) == 2 and a._pooled
    s, p = pool.acquire([1, 2, 3, 4, 5, 7, 8])
    assert p == 5 and s.slot == 3 and not s.prefilled and s._prefill_from == 5 and s._dprefill_from == 0
    fresh, p0 = pool.acquire([5, 5, 5])
    assert p0 == 0 and fresh.slot is None
    c = batching.Session(e, [7], temperature=0.0)
    c.slot = 6
    d = batching.Session(e, [8], temperature=0.0)
    d.slot = 7
    pool.put(c)
    pool.put(d)                          # over max_pooled: the oldest frees its slot
    assert e._runner.released == [4]


def test_grammar_and_empty_prompt_rejected():
    e = _Engine()
    with pytest.raises(NotImplementedError):
        batching.Session(e, [1], grammar=object())
    with pytest.raises(ValueError):
        batching.Session(e, [])
