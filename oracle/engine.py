"""Oracle (test infrastructure): restatement of the androidllm decode loop.

``OracleEngine`` follows ``LayerStreamingEngine`` (``androidllm/engine.py``)
with every layer resident (the reference's ``keep_layers = n_layers`` case):
streaming, LRU, layer skipping, throttling, grammar masking and prefix reuse
are not on the speculative-decode path and are left out.  Sampling draws from
a numpy Generator exactly like ``engine.py:278-286`` (``_sample``, since the
Rust sampler is not importable) so a seeded run reproduces the reference.
With ``sampler="fixed"`` every sample is ``sampling.sample_fixed`` on the
generator's next uniform draw instead (the device sampler's arithmetic; the
same draws in the same order as ``rng.choice``).
"""
import numpy as np

from . import io, llama, sampling


class OracleEngine:
    def __init__(self, model_dir, draft_dir=None, spec_k=0, seed=None, sampler="reference"):
        canon, embed, fnorm, head, layers = io.load_model(model_dir)
        self.canon = canon
        self.model = llama.OracleModel(canon, embed, fnorm, head)
        self.layers = layers
        self.n_layers = canon["layers"]
        self.ctx_len = min(int(canon["max_len"]), 4096)          # engine.py:119-120
        self.rng = np.random.default_rng(seed)
        self.sampler = sampler
        self.spec_k = max(0, int(spec_k))
        self.draft = OracleEngine(draft_dir) if draft_dir else None
        self.stats = {"tokens_served": 0, "draft_tokens": 0, "spec_accepted": 0,
                      "spec_bonus": 0, "spec_steps": 0}
        self.trace = []   # (kind, logits) of every sampled position, for margins

    def _sample(self, lg, temperature, top_p, min_p):
        if self.sampler == "fixed":
            if temperature <= 0:
                return int(np.argmax(np.asarray(lg, dtype=np.float32).reshape(-1)))
            return sampling.sample_fixed(lg, temperature, top_p, min_p, self.rng.random())
        return sampling.sample_reference(lg, temperature, top_p, min_p, self.rng)

    # engine.py:255-264
    def _forward(self, x, kv, pos):
        for li, layer in enumerate(self.layers):
            x = self.model.layer_forward(x, layer, kv[li], pos)
        return x

    def _score(self, x):
        return self.model.logits(x)

    # engine.py:278-286 (no grammar)
    def _step(self, kv, pos, token, temperature, top_p, min_p, record=None):
        x = self._forward(self.model.embed[token].reshape(1, self.model.hidden), kv, pos)
        lg = self._score(x)
        if record is not None:
            record.append(lg)
        return self._sample(lg, temperature, top_p, min_p)

    # engine.py:288-320
    def _spec_step(self, kv, dkv, pos, token, temperature, top_p, min_p):
        d = self.draft
        cands = []
        dtok, dpos = token, pos
        for _ in range(self.spec_k):
            dx = d._forward(d.model.embed[dtok].reshape(1, d.model.hidden), dkv, dpos)
            cands.append(self._sample(d._score(dx), temperature, top_p, min_p))
            dtok = cands[-1]
            dpos += 1
        self.stats["draft_tokens"] += self.spec_k
        emitted = []
        tpos, tok = pos, token
        for c in cands:
            g = self._step(kv, tpos, tok, temperature, top_p, min_p, self.trace)
            if g == c:
                emitted.append(c)
                tok = c
                tpos += 1
            else:
                emitted.append(g)
                return emitted, g, tpos + 1, len(emitted) - 1
        g = self._step(kv, tpos, tok, temperature, top_p, min_p, self.trace)
        emitted.append(g)
        return emitted, g, tpos + 1, len(emitted) - 1

    # engine.py:322-405 (spec and plain branches; no grammar / prefix reuse)
    def generate(self, prompt_ids, max_new_tokens=64, temperature=0.8, top_p=0.9,
                 min_p=0.0, stop_ids=()):
        prompt_ids = list(prompt_ids)[: self.ctx_len]
        kv = self.model.prepare_kv(self.ctx_len)
        spec = self.draft is not None and self.spec_k > 0
        for i in range(len(prompt_ids) - 1):
            self._forward(self.model.embed[prompt_ids[i]].reshape(1, self.model.hidden), kv, i)
        token = prompt_ids[-1]
        pos = len(prompt_ids) - 1
        if spec:
            dkv = self.draft.model.prepare_kv(self.ctx_len)
            for i, t in enumerate(prompt_ids):
                self.draft._forward(self.draft.model.embed[t].reshape(1, self.draft.model.hidden),
                                    dkv, i)
        out = []
        while len(out) < max_new_tokens:
            if token in stop_ids:
                break
            if spec:
                emitted, token, pos, n_draft = self._spec_step(kv, dkv, pos, token,
                                                               temperature, top_p, min_p)
                self.stats["spec_steps"] += 1
                for i, t in enumerate(emitted):
                    if t in stop_ids:
                        token = t
                        break
                    if len(out) >= max_new_tokens:
                        break
                    out.append(t)
                    self.stats["tokens_served"] += 1
                    self.stats["spec_accepted" if i < n_draft else "spec_bonus"] += 1
                if len(out) >= max_new_tokens:
                    break
            else:
                token = self._step(kv, pos, token, temperature, top_p, min_p, self.trace)
                pos += 1
                if token in stop_ids:
                    break
                out.append(token)
                self.stats["tokens_served"] += 1
        return out
