"""Continuous batching of chat sessions on the device.

The reference (androidllm/batching.py) serves concurrent requests with one
scheduler thread that round-robins ONE session's work unit per visit (a
prefill chunk or one decode / speculative step), so N sessions share the
device by time-slicing and every step streams all of a model's weights for a
single sequence.  Here the scheduler advances every active session in the
same visit:

* each session owns a slot of a multi-slot paged KV cache (16-position
  pages, one page-table row per slot) for the target and one for the draft;
* a speculative step of B sessions runs the k draft forwards as k
  multi-sequence passes of B rows (one per session) and the verification as
  passes of up to 64 rows (k + 1 per session; alm_model_max_pass_rows): the
  weights stream once per pass for all its sessions (alm_forward_seqs);
* prompts are prefilled into their slots in chunks of up to 256 rows
  through the dense path (alm_prefill_slot).

Each session's tokens equal what LayerStreamingEngine.generate returns for it
alone: rows never mix in a reduction, and a session with temperature > 0
draws its uniforms from its own generator in the reference's order (k draft
draws, then one per verified row up to the first rejection, then the bonus;
androidllm/engine.py:288-320).  The reference's sessions share the engine's
generator, so its draws depend on the visiting order.

Session, SessionPool and BatchScheduler keep the reference's names,
arguments and snapshot keys.  Differences: a pooled session with a longer
new prompt prefills the part after the shared prefix (the reference's
reuse_kv skips it, batching.py:62-69) and refills its draft cache from
position 0; grammar-constrained sessions are rejected like in the engine.
"""
import contextlib
import os
import threading
import time
from collections import deque

import numpy as np

from .ops import DeviceKV

MAX_PASS_SEQS = 16   # sequences of one multi-sequence pass


def kv_bytes_per_session(engine, ctx_len=None):
    """Per-session KV cache size: layers * kv_heads * head_dim * (k+v) * 2 B
    per position (androidllm/batching.py:22-28)."""
    ctx = ctx_len or engine.ctx_len
    c = engine.canon
    return ctx * c["kv_heads"] * c["head_dim"] * 2 * 2 * c["layers"]


class BatchRunner:
    """The device side: slot KV caches of the target (and draft) and the
    batched steps over sessions."""

    def __init__(self, engine, slots=4):
        if slots < 1:
            raise ValueError("slots must be positive")
        self.engine = engine
        self.slots = int(slots)
        self.cap = engine.ctx_len + engine.spec_k + 1
        self.tkv = DeviceKV(engine.dm, self.cap, 16, slots=self.slots)
        self.draft = engine.draft
        self.dkv = DeviceKV(self.draft.dm, self.cap, 16, slots=self.slots) if self.draft is not None else None
        self.pass_rows = engine.dm.max_pass_rows()
        self._free = list(range(self.slots))
        self._lock = threading.Lock()

    def acquire_slot(self):
        with self._lock:
            if not self._free:
                raise RuntimeError("no free KV slot")
            return self._free.pop(0)

    def release_slot(self, slot):
        with self._lock:
            if slot is not None and slot not in self._free:
                self._free.append(slot)

    def free_slots(self):
        with self._lock:
            return len(self._free)

    def close(self):
        for kv in (self.tkv, self.dkv):
            if kv is not None:
                kv.close()

    # -- decode -----------------------------------------------------------------------
    def step(self, sessions):
        """One decode work unit for every session (all prefilled, not done)."""
        spec = [s for s in sessions if s.using_spec]
        plain = [s for s in sessions if not s.using_spec]
        if spec:
            self._spec_steps(spec)
        if plain:
            self._plain_steps(plain)

    @staticmethod
    def _picks(model, am, parts):
        """The tokens of a pass's sequences: parts = [(session, rows, draws)]
        in row order; greedy sessions take the pass's argmax rows, sampling
        sessions the device sampler, one call per run of consecutive sessions
        with the same settings."""
        out, row0, i = [], 0, 0
        while i < len(parts):
            s, n, u = parts[i]
            if not s.temperature > 0:
                out.append([int(t) for t in am[i]])
                row0 += n
                i += 1
                continue
            j, rows, us = i, 0, []
            key = (s.temperature, s.top_p, s.min_p)
            while j < len(parts) and parts[j][0].temperature > 0 and \
                    (parts[j][0].temperature, parts[j][0].top_p, parts[j][0].min_p) == key:
                rows += parts[j][1]
                us.append(parts[j][2])
                j += 1
            picks = model.sample_rows(row0, rows, s.temperature, s.top_p, s.min_p, np.concatenate(us))
            k = 0
            for p in parts[i:j]:
                out.append([int(t) for t in picks[k:k + p[1]]])
                k += p[1]
            row0 += rows
            i = j
        return out

    def _plain_steps(self, sessions):
        dm = self.engine.dm
        for i in range(0, len(sessions), MAX_PASS_SEQS):
            group = sessions[i:i + MAX_PASS_SEQS]
            for s in group:
                s._ensure_draws(1)
            _, am = dm.forward_seqs(self.tkv, [(s.slot, [s.token], s.pos) for s in group])
            picks = self._picks(dm, am, [(s, 1, s._draws(1)) for s in group])
            for s, p in zip(group, picks):
                s._consume(1)
                s._advance([p[0]], 0)

    def _spec_steps(self, sessions):
        e, d = self.engine, self.draft.dm
        K = e.spec_k
        for s in sessions:
            s._ensure_draws(2 * K + 1)
        # draft: K passes of one row per session
        cands = {id(s): [] for s in sessions}
        dtok = {id(s): s.token for s in sessions}
        for j in range(K):
            for i in range(0, len(sessions), MAX_PASS_SEQS):
                group = sessions[i:i + MAX_PASS_SEQS]
                _, am = d.forward_seqs(self.dkv, [(s.slot, [dtok[id(s)]], s.pos + j) for s in group])
                parts = []
                for s in group:
                    u = s._draws(K)
                    parts.append((s, 1, None if u is None else u[j:j + 1]))
                for s, p in zip(group, self._picks(d, am, parts)):
                    cands[id(s)].append(p[0])
                    dtok[id(s)] = p[0]
        e.stats["draft_tokens"] = e.stats.get("draft_tokens", 0) + K * len(sessions)
        # verify: k + 1 rows per session, as many sessions per pass as fit
        dm = e.dm
        per = max(1, min(MAX_PASS_SEQS, self.pass_rows // (K + 1)))
        for i in range(0, len(sessions), per):
            group = sessions[i:i + per]
            _, am = dm.forward_seqs(self.tkv, [(s.slot, [s.token] + cands[id(s)], s.pos) for s in group])
            parts = []
            for s in group:
                u = s._draws(2 * K + 1)
                parts.append((s, K + 1, None if u is None else u[K:]))
            for s, picks in zip(group, self._picks(dm, am, parts)):
                c = cands[id(s)]
                emitted = []
                for k in range(K):
                    emitted.append(picks[k])
                    if picks[k] != c[k]:
                        break
                else:
                    emitted.append(picks[K])
                n_acc = len(emitted) - 1
                s._consume(K + n_acc + 1)
                s._advance(emitted, n_acc)
                e.stats["spec_steps"] = e.stats.get("spec_steps", 0) + 1


class Session:
    """One generation in progress (androidllm/batching.py:31-149).
    Invariant: the slot's KV holds positions 0..pos-1, token = id at pos."""

    def __init__(self, engine, prompt_ids, max_new_tokens=64, temperature=0.8, top_p=0.9, min_p=0.0,
                 stop_ids=(), grammar=None, prefill_chunk=256, seed=None):
        if grammar is not None:
            raise NotImplementedError("grammar-constrained decoding is outside this engine")
        self.engine = engine
        self.prompt_ids = [int(t) for t in list(prompt_ids)[: engine.ctx_len]]
        if not self.prompt_ids:
            raise ValueError("empty prompt")
        self.max_new_tokens = int(max_new_tokens)
        self.temperature = temperature
        self.top_p = top_p
        self.min_p = min_p
        self.stop_ids = tuple(stop_ids)
        self.grammar = None
        self.prefill_chunk = max(1, int(prefill_chunk))
        self.slot = None
        self.pos = 0
        self.token = None
        self.prefilled = False
        self.done = False
        self.generated = []
        self.buf_parts = []
        self.error = None
        self.started = time.time()
        self.using_spec = engine.draft is not None and engine.spec_k > 0
        self._prefill_from = 0
        self._dprefill_from = 0
        self._pooled = False
        self._rng = np.random.default_rng(seed)
        self._u = np.empty(0, np.float64)
        self._u_used = 0
        self._kv_ids = []            # tokens whose KV the slot holds (prefix reuse)

    # -- uniforms (the session's own stream, consumed in the reference's order) ------
    def _ensure_draws(self, n):
        if self.temperature > 0 and self._u.size - self._u_used < n:
            self._u = np.concatenate([self._u[self._u_used:], self._rng.random(max(4096, n))])
            self._u_used = 0

    def _draws(self, n):
        if not self.temperature > 0:
            return None
        return self._u[self._u_used:self._u_used + n]

    def _consume(self, n):
        if self.temperature > 0:
            self._u_used += n

    # -- pool reuse ------------------------------------------------------------------
    def reuse_kv(self, pfx):
        """Continue from a pooled slot that holds prompt[0..pfx-1]: the
        target's prefill resumes at pfx; the draft's cache is refilled from 0
        (a draft cache can miss the last candidate of an all-accept step,
        androidllm/engine.py:299-303)."""
        self.prefilled = False
        self._prefill_from = int(pfx)
        self._dprefill_from = 0
        self.pos = int(pfx)

    def common_prefix(self, other_ids):
        n = min(len(self._kv_ids), len(other_ids), self.engine.ctx_len)
        p = 0
        while p < n and self._kv_ids[p] == other_ids[p]:
            p += 1
        return p

    # -- work units ------------------------------------------------------------------
    def _runner(self):
        return self.engine.batch_runner()

    def _prefill_unit(self, runner):
        """Prefill the next chunk of the prompt (target up to the last prompt
        token, the draft through it)."""
        ids = self.prompt_ids
        start = self._prefill_from
        end = min(start + self.prefill_chunk, len(ids) - 1)
        if end > start:
            self.engine.dm.prefill(runner.tkv, ids[start:end], start, slot=self.slot)
        if self.using_spec:
            dstart = self._dprefill_from
            dend = min(dstart + self.prefill_chunk, len(ids))
            if end >= len(ids) - 1:
                dend = len(ids)          # the draft also holds the last prompt token
            if dend > dstart:
                runner.draft.dm.prefill(runner.dkv, ids[dstart:dend], dstart, slot=self.slot)
            self._dprefill_from = dend
        self._prefill_from = end
        if end >= len(ids) - 1:
            self.pos = len(ids) - 1
            self.token = ids[-1]
            self.prefilled = True
            self._kv_ids = list(ids[:-1])

    def _check_budget(self):
        if len(self.generated) >= self.max_new_tokens or self.token in self.stop_ids:
            self.done = True
        return self.done

    def _advance(self, emitted, n_draft):
        """Take a step's emitted tokens (androidllm/batching.py:93-109)."""
        e = self.engine
        self._kv_ids.extend([self.token] + list(emitted[:-1]))
        self.pos += len(emitted)
        self.token = emitted[-1]
        new = []
        for i, t in enumerate(emitted):
            if t in self.stop_ids:
                self.token = t
                self.done = True
                break
            if len(self.generated) >= self.max_new_tokens:
                break
            self.generated.append(t)
            new.append(t)
            e.stats["tokens_served"] += 1
            if self.using_spec:
                key = "spec_accepted" if i < n_draft else "spec_bonus"
                e.stats[key] = e.stats.get(key, 0) + 1
        if len(self.generated) >= self.max_new_tokens:
            self.done = True
        self._new = new

    def step(self):
        """Advance one work unit on its own. Returns (finished, new_tokens)."""
        finished, new = advance([self])[0]
        return finished, new


def advance(sessions):
    """One work unit for each session: a prefill chunk for sessions still
    prefilling (one slot each), one batched decode step for all the others.
    Returns [(finished, new_tokens)] in the given order."""
    if not sessions:
        return []
    runner = sessions[0].engine.batch_runner()
    out = {}
    decode = []
    for s in sessions:
        if s.done:
            out[id(s)] = (True, [])
            continue
        if s.slot is None:
            s.slot = runner.acquire_slot()
        if not s.prefilled:
            s._prefill_unit(runner)
            out[id(s)] = (False, [])
            continue
        if s._check_budget():
            out[id(s)] = (True, [])
            continue
        decode.append(s)
    for s in decode:
        s._new = []
    if decode:
        runner.step(decode)
    for s in decode:
        out[id(s)] = (s.done, list(s._new))
    return [out[id(s)] for s in sessions]


class SessionPool:
    """Finished sessions kept with their KV slots for prefix reuse
    (androidllm/batching.py:150-198): acquire pops the one whose cached
    tokens share the longest prefix with the new prompt."""

    def __init__(self, engine, max_pooled=4):
        self.engine = engine
        self.max_pooled = max_pooled
        self._sessions = []
        self._lock = threading.Lock()

    def acquire(self, prompt_ids):
        with self._lock:
            best, best_p = None, 1
            for i, s in enumerate(self._sessions):
                p = s.common_prefix(list(prompt_ids))
                if p > best_p:
                    best_p, best = p, i
            if best is None:
                return Session(self.engine, prompt_ids), 0
            old = self._sessions.pop(best)
        s = Session(self.engine, prompt_ids)
        s.slot = old.slot
        s._kv_ids = old._kv_ids[:best_p]
        s.reuse_kv(min(best_p, len(s.prompt_ids) - 1))
        return s, best_p

    def put(self, sess):
        if sess.error or sess.slot is None:
            return
        sess._pooled = True
        with self._lock:
            self._sessions.append(sess)
            if len(self._sessions) > self.max_pooled:
                old = self._sessions.pop(0)
                self.engine.batch_runner().release_slot(old.slot)

    def __len__(self):
        with self._lock:
            return len(self._sessions)


class BatchScheduler:
    """Scheduler thread (androidllm/batching.py:200-272): submit() returns
    True when a slot was taken; each visit advances every active session by
    one work unit, decode steps batched across sessions; the done callback
    fires on the scheduler thread."""

    def __init__(self, engine, max_slots=4):
        self.engine = engine
        kv = kv_bytes_per_session(engine)
        budget = int(os.environ.get("ANDROIDLLM_BATCH_MEM_MB", "700")) * 1048576
        cap = max(1, budget // max(kv, 1))
        self.max_slots = min(max(1, int(max_slots)), cap, engine.batch_runner().slots)
        self._active = deque()
        self._cond = threading.Condition()
        self._stop = False
        self.stats = {"active": 0, "queued": 0, "max": self.max_slots, "completed": 0, "stepped": 0,
                      "rejected": 0}
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def submit(self, session, done_cb):
        with self._cond:
            if len(self._active) >= self.max_slots:
                self.stats["rejected"] += 1
                return False
            self._active.append((session, done_cb))
            self.stats["queued"] += 1
            self._cond.notify()
        return True

    def active_count(self):
        with self._cond:
            return len(self._active)

    def close(self):
        with self._cond:
            self._stop = True
            self._cond.notify_all()
        self._thread.join(timeout=30)

    def _run(self):
        runner = self.engine.batch_runner()
        while True:
            with self._cond:
                while not self._active and not self._stop:
                    self._cond.wait()
                if self._stop:
                    return
                slots = list(self._active)
            sessions = [s for s, _ in slots]
            try:
                results = advance(sessions)
            except Exception as exc:
                results = []
                for s in sessions:
                    s.error = str(exc)
                    s.done = True
                    results.append((True, []))
            self.stats["stepped"] += len(sessions)
            finished = [(slot, r[0]) for slot, r in zip(slots, results)]
            with self._cond:
                for (sess, cb), fin in finished:
                    if fin:
                        self._active.remove((sess, cb))
                        self.stats["queued"] = max(0, self.stats["queued"] - 1)
                        self.stats["completed"] += 1
            for (sess, cb), fin in finished:
                if fin:
                    with contextlib.suppress(Exception):
                        cb(sess)
                    if not sess._pooled:      # the callback did not keep it in a SessionPool
                        runner.release_slot(sess.slot)
                        sess.slot = None

    def snapshot(self):
        with self._cond:
            return {"active": len(self._active), "queued": self.stats["queued"], "max": self.max_slots,
                    "completed": self.stats["completed"], "rejected": self.stats["rejected"]}


def run_batch(engine, prompts, max_new_tokens=64, temperature=0.0, top_p=0.9, min_p=0.0, seeds=None,
              stop_ids=(), max_active=None):
    """Generate for every prompt (no thread): at most ``max_active``
    sessions (default: all) advance together; a finished session frees its
    slot for the next prompt in line (continuous batching).  Returns the
    token lists in prompt order and frees the slots."""
    outs = _broadcast(max_new_tokens, len(prompts))
    sessions = [Session(engine, p, max_new_tokens=m, temperature=temperature, top_p=top_p, min_p=min_p,
                        stop_ids=stop_ids, seed=None if seeds is None else seeds[i])
                for i, (p, m) in enumerate(zip(prompts, outs))]
    runner = engine.batch_runner()
    cap = min(len(sessions), int(max_active or len(sessions)), runner.slots)
    queue = deque(sessions)
    active = []
    try:
        while queue or active:
            while queue and len(active) < cap:
                active.append(queue.popleft())
            res = advance(active)
            still = []
            for s, (fin, _) in zip(active, res):
                if fin:
                    runner.release_slot(s.slot)
                    s.slot = None
                else:
                    still.append(s)
            active = still
    finally:
        for s in sessions:
            runner.release_slot(s.slot)
            s.slot = None
    return [s.generated for s in sessions]


def _broadcast(v, n):
    return list(v) if isinstance(v, (list, tuple)) else [v] * n


__all__ = ["BatchRunner", "BatchScheduler", "Session", "SessionPool", "advance", "kv_bytes_per_session",
           "run_batch", "MAX_PASS_SEQS"]
