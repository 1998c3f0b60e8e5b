"""HBM-resident drop-in for androidllm's LayerStreamingEngine.

Same constructor, ``generate`` / ``_spec_step`` / ``_step`` / ``_forward`` /
``snapshot`` surface as ``androidllm/engine.py:75-459``, with the layer
streaming replaced by weights that stay resident in HBM (the whole point of
streaming was a phone's RAM; a B200 holds the model many times over):

* the shard directory is read once and uploaded without host dequantization;
* a decode step is one device forward (embedding, every layer, final norm,
  head, argmax) and a speculative step — K draft forwards, one (K+1)-row
  verify forward of the target and the acceptance — is one CUDA-graph replay
  with no host round trip inside it;
* acceptance follows ``engine.py:306-320``: accept while the target's pick
  equals the draft's candidate, then emit the target's correction, or a
  bonus token after K accepts.  At temperature > 0 both picks are samples
  (``engine.py:26-45`` on the device, ``alm_sample``'s fixed arithmetic)
  driven by one stream of uniform draws consumed in the reference's order:
  the K draft samples, then one per verified target row up to the first
  rejection; a plain step takes one draw.

The target's cache keeps the longest common prefix with the previous prompt
(``engine.py:245-253``; ``ANDROIDLLM_PREFIX_KV=0`` turns it off, as in the
reference).  Not in the reference: ``seed`` makes the draw stream
reproducible (the reference's generator is unseeded); ``draft_refresh=True``
has the draft forward the token before each step's position again, which
repairs the draft's stale cache entry after a step that accepted every
candidate; ``accept_rule="rejection"`` accepts sampled candidates by
speculative rejection sampling (u < min(1, p/q), the residual max(0, p - q)
resampled at the first rejection, 2k + 1 draws per step).  Out of the path
and not carried over: layer skipping, throttling, grammar masking (grammar
disables speculation in the reference too) and the tokenizer.
"""
import os
import time

import numpy as np

from . import quant
from .models.llama import KVList, LlamaModel
from .ops import DeviceKV, DeviceModel, SpecDecoder, default_context, load_manifest
from . import safetensors



class LayerStreamingEngine:
    def __init__(self, model_dir, keep_layers=0, draft_dir=None, spec_k=0, device=0, seed=None,
                 accept_rule="reference", draft_refresh=False, _ctx=None):
        if accept_rule not in ("reference", "rejection"):
            raise ValueError("accept_rule must be 'reference' or 'rejection'")
        self.accept_rule = accept_rule
        self.draft_refresh = bool(draft_refresh)
        self.model_dir = model_dir
        self.manifest = load_manifest(model_dir)
        canon = self.manifest["config"]
        self.canon = canon
        self.n_layers = canon["layers"]
        self.layer_meta = self.manifest.get("quant", {}).get("layers", {})
        self.ctx = _ctx or default_context(device)
        t0 = time.time()
        self.dm = DeviceModel.from_dir(self.ctx, model_dir)
        load_ms = (time.time() - t0) * 1000
        self.model = LlamaModel.from_device(self.dm, embed=_EmbedRows(model_dir, self.manifest))
        self.ctx_len = min(int(canon["max_len"]), int(os.environ.get("ANDROIDLLM_MAX_CTX", "4096")))
        self._keep = self.n_layers
        self._rng = np.random.default_rng(seed)
        self._u = np.empty(0, np.float64)   # drawn uniforms; self._u[self._u_used:] not consumed yet
        self._u_used = 0
        self._u_host_moved = False          # the host consumed draws after the last upload
        self.stats = {"cache_hits": 0, "cache_misses": self.n_layers, "load_ms": load_ms,
                      "load_calls": self.n_layers, "compute_ms": 0.0, "compute_tokens": 0,
                      "tokens_served": 0, "prefix_calls": 0, "prefix_tokens": 0,
                      "started": time.time()}
        self.draft = None
        self.spec_k = max(0, int(spec_k))
        if draft_dir:
            self.draft = LayerStreamingEngine(draft_dir, _ctx=self.ctx)
            self.draft.spec_k = 0
        self.tokenizer = None
        self.stop_ids = ()
        self._kv = None
        self._spec = None
        self._kv_len = 0
        self._kv_prompt_ids = None
        self._prefix_kv = os.environ.get("ANDROIDLLM_PREFIX_KV", "1") not in ("0", "false", "")

    # -- caches --------------------------------------------------------------------
    def batch_runner(self, slots=None):
        """The device side of batched sessions (androidllm_b200.batching):
        slot KV caches for ``slots`` concurrent sessions (default
        ANDROIDLLM_BATCH_MAX, else 8), created on first use."""
        if getattr(self, "_batch", None) is None:
            from .batching import BatchRunner
            n = int(slots or os.environ.get("ANDROIDLLM_BATCH_MAX", "8"))
            self._batch = BatchRunner(self, slots=n)
        return self._batch

    def generate_batch(self, prompts, max_new_tokens=64, temperature=0.8, top_p=0.9, min_p=0.0, seeds=None,
                       stop_ids=(), max_active=None):
        """Generate for several prompts at once (every active session advances
        in each step, the weights stream once per pass for all of them; at
        most max_active at a time, the rest queued); each result equals
        generate() for that prompt alone (with seeds[i] as the engine's seed
        when sampling)."""
        from .batching import run_batch
        return run_batch(self, prompts, max_new_tokens, temperature, top_p, min_p, seeds, stop_ids, max_active)

    def _kv_capacity(self):
        return self.ctx_len + self.spec_k + 1

    def _target_kv(self):
        if self._kv is None:
            self._kv = KVList(DeviceKV(self.dm, self._kv_capacity()), self.n_layers)
        return self._kv

    def _draft_kv(self):
        d = self.draft
        if d._kv is None:
            d._kv = KVList(DeviceKV(d.dm, self._kv_capacity()), d.n_layers)
        return d._kv

    def _spec_decoder(self):
        if self._spec is None:
            self._spec = SpecDecoder(self.dm, self.draft.dm, self._target_kv().cache, self._draft_kv().cache,
                                     self.spec_k)
        self._spec.set_draft_refresh(self.draft_refresh)
        return self._spec

    def _match_prefix(self, ids):
        """engine.py:245-253: common prefix length with the previous prompt."""
        if not self._prefix_kv or self._kv is None or not self._kv_prompt_ids:
            return 0
        old = self._kv_prompt_ids
        n = min(len(old), len(ids), self.ctx_len)
        p = 0
        while p < n and old[p] == ids[p]:
            p += 1
        return p

    @staticmethod
    def _begin(dec, prev, token, pos):
        """Set the decoder's state: token at pos, and the token at pos - 1
        (which the draft refresh forwards again) when there is one."""
        if prev is None or pos < 1:
            dec.begin(token, pos)
        else:
            dec.begin(token, pos, prev=int(prev))

    # -- reference-compatible pieces --------------------------------------------------
    def load_layer(self, i):
        """The resident layer i (shard-format projections + norms)."""
        self.stats["cache_hits"] += 1
        return self.dm._layer_src[i]

    def _forward(self, x, kv, pos):
        """engine.py:255-264: one full pass at pos (rows of x = consecutive positions)."""
        t0 = time.time()
        for li in range(self.n_layers):
            x = self.model.layer_forward(x, self.load_layer(li), kv[li], pos)
        self._account(t0, np.asarray(x).reshape(-1, self.canon["hidden"]).shape[0])
        return x

    def _score(self, x):
        return self.model.logits(x)

    def _account(self, t0, rows):
        self.stats["compute_ms"] += (time.time() - t0) * 1000
        self.stats["compute_tokens"] += self.n_layers * rows

    def _prefill(self, kv, ids, pos0):
        """The prompt's KV entries (androidllm/engine.py:345-361), in chunks of
        up to 256 rows through the dense path (DeviceModel.prefill)."""
        t0 = time.time()
        self.dm.prefill(kv.cache, ids, pos0)
        self._account(t0, len(ids))

    # -- uniform draws (one stream, consumed in the reference's order) ---------------
    def _draws(self, n):
        """Make at least n unconsumed draws available in self._u."""
        if self._u.size - self._u_used < n:
            self._u = np.concatenate([self._u[self._u_used:], self._rng.random(max(4096, n))])
            self._u_used = 0

    def _next_draw(self):
        self._draws(1)
        u = float(self._u[self._u_used])
        self._u_used += 1
        self._u_host_moved = True
        return u

    def _feed_spec(self, dec, temperature, top_p, min_p):
        """Sampling settings and enough draws for one speculative step."""
        dec.set_sampling(temperature, top_p, min_p)
        dec.set_rejection(self.accept_rule == "rejection" and temperature > 0)
        if temperature > 0:
            need = 2 * self.spec_k + 1
            if dec._uniforms is not self._u or self._u_host_moved or self._u.size - self._u_used < need:
                self._draws(need)
                dec.set_uniforms(self._u[self._u_used:])
                self._u = dec._uniforms
                self._u_used = 0
                self._u_host_moved = False

    def _step(self, kv, pos, token, temperature, top_p, min_p, grammar=None, buf_parts=None):
        """engine.py:278-286: embed, full forward at pos, pick the next token."""
        _check_grammar(grammar)
        t0 = time.time()
        _, am = self.dm.forward(kv.cache, [token], pos)
        self._account(t0, 1)
        if temperature > 0:
            return int(self.dm.sample(1, temperature, top_p, min_p, [self._next_draw()])[0])
        return int(am[0])

    def _spec_step(self, kv, dkv, pos, token, temperature, top_p, min_p):
        """engine.py:288-320 on the device: returns (emitted, next_token,
        next_pos, n_draft_accepted)."""
        s = self._spec_decoder()
        if kv is not self._kv or dkv is not self.draft._kv:
            raise ValueError("speculative steps run on the engine's own KV caches")
        self._feed_spec(s, temperature, top_p, min_p)
        s.begin(token, pos)
        t0 = time.time()
        emitted, acc = s.run(1)
        if temperature > 0:
            self._u_used = s.uniforms_used()
        self._account(t0, self.spec_k + 1)
        self.draft._account(t0, self.spec_k)
        self.stats["draft_tokens"] = self.stats.get("draft_tokens", 0) + self.spec_k
        return emitted, emitted[-1], pos + len(emitted), acc[0]

    # -- generate ---------------------------------------------------------------------
    def generate(self, prompt_ids, max_new_tokens=64, temperature=0.8, top_p=0.9, min_p=0.0,
                 stop_ids=(), callback=None, grammar=None):
        _check_grammar(grammar)
        prompt_ids = [int(t) for t in list(prompt_ids)[: self.ctx_len]]
        if not prompt_ids:
            raise ValueError("empty prompt")
        kv = self._target_kv()
        # prompt-prefix reuse across calls (engine.py:245-253, 325-336): the
        # target's cache keeps the positions of the longest common prefix
        # with the previous prompt and prefill starts after it
        pfx = self._match_prefix(prompt_ids)
        if pfx > 1:
            start = pfx
            self.stats["prefix_calls"] += 1
            self.stats["prefix_tokens"] += pfx
        else:
            kv.cache.zero()
            start = 0
        self._kv_prompt_ids = prompt_ids
        spec = self.draft is not None and self.spec_k > 0
        if spec:
            for k in ("draft_tokens", "spec_accepted", "spec_bonus", "spec_steps"):
                self.stats.setdefault(k, 0)
        # prefill: kv[0..n-2] filled, token = id at position n-1 (engine.py:346-354)
        t_pre = time.perf_counter()
        if start < len(prompt_ids) - 1:
            self._prefill(kv, prompt_ids[start:-1], start)
        token = prompt_ids[-1]
        pos = len(prompt_ids) - 1
        if spec:
            dkv = self._draft_kv()
            dkv.cache.zero()
            self.draft._prefill(dkv, prompt_ids, 0)
            dec = self._spec_decoder()
        prev = prompt_ids[-2] if len(prompt_ids) >= 2 else None
        if spec:
            self._begin(dec, prev, token, pos)
        t_pre = time.perf_counter() - t_pre
        generated = []
        steps = 0
        t_dec = time.perf_counter()
        while len(generated) < max_new_tokens:
            if token in stop_ids:
                break
            if spec:
                # one speculative step: the step's input state goes to the
                # device, its emitted tokens come back (engine.py:369-387)
                t0 = time.time()
                self._feed_spec(dec, temperature, top_p, min_p)
                self._begin(dec, prev, token, pos)
                emitted, accepted = dec.run(1)
                if temperature > 0:
                    self._u_used = dec.uniforms_used()
                self._account(t0, self.spec_k + 1)
                self.draft._account(t0, self.spec_k)
                n_draft = accepted[0]
                prev = emitted[-2] if len(emitted) >= 2 else token
                token = emitted[-1]
                pos += len(emitted)
                steps += 1
                self.stats["spec_steps"] += 1
                self.stats["draft_tokens"] += self.spec_k
                for i, t in enumerate(emitted):
                    if t in stop_ids:
                        token = t
                        break
                    if len(generated) >= max_new_tokens:
                        break
                    generated.append(t)
                    self.stats["tokens_served"] += 1
                    self.stats["spec_accepted" if i < n_draft else "spec_bonus"] += 1
                    if callback:
                        callback(t)
                if len(generated) >= max_new_tokens:
                    break
            else:
                token = self._step(kv, pos, token, temperature, top_p, min_p)
                pos += 1
                steps += 1
                if token in stop_ids:
                    break
                generated.append(token)
                self.stats["tokens_served"] += 1
                if callback:
                    callback(token)
        self.last_decode = {"seconds": time.perf_counter() - t_dec, "prefill_seconds": t_pre, "tokens": len(generated),
                            "steps": steps}
        self._kv_len = pos
        return generated

    def close(self):
        if getattr(self, "_batch", None) is not None:
            self._batch.close()
            self._batch = None
        if self._spec is not None:
            self._spec.close()
            self._spec = None
        if self.draft is not None:
            self.draft.close()
            self.draft = None

    def snapshot(self):
        """engine.py:417-459 keys."""
        up = time.time() - self.stats["started"]
        snap = {
            "model": self.manifest.get("name", "androidllm"),
            "uptime_s": int(up),
            "tokens_served": self.stats["tokens_served"],
            "cache_hits": self.stats["cache_hits"],
            "cache_misses": self.stats["cache_misses"],
            "cache_size": self.n_layers,
            "keep_layers": self._keep,
            "lru_layers": 0,
            "skip_every": 0,
            "ctx_len": self.ctx_len,
            "prefix_kv": self._prefix_kv,
            "prefix_calls": self.stats["prefix_calls"],
            "prefix_tokens": self.stats["prefix_tokens"],
            "context_used": self._kv_len,
            "context_pct": round(self._kv_len / self.ctx_len * 100, 1) if self.ctx_len else 0.0,
            "paused": False,
            "throttle_ms": 0,
            "load_ms_avg": self.stats["load_ms"] / max(1, self.stats["load_calls"]),
            "compute_ms_per_token": (self.stats["compute_ms"] / self.stats["compute_tokens"]
                                     if self.stats["compute_tokens"] else 0.0),
            "rss_mb": 0.0,
        }
        if self.draft is not None:
            acc = self.stats.get("spec_accepted", 0)
            bon = self.stats.get("spec_bonus", 0)
            snap["spec"] = {
                "enabled": self.spec_k > 0,
                "k": self.spec_k,
                "draft": self.draft.manifest.get("name", "draft"),
                "steps": self.stats.get("spec_steps", 0),
                "draft_tokens": self.stats.get("draft_tokens", 0),
                "accepted": acc,
                "bonus": bon,
                "accept_rate": round(acc / (acc + bon), 3) if (acc + bon) else 0.0,
            }
        return snap


def _check_grammar(grammar):
    if grammar is not None:
        raise NotImplementedError("grammar-constrained decoding is outside this engine")


class _EmbedRows:
    """``model.embed[token]`` of the reference: fp16 rows of the shard's
    embedding table (int8 per-row dequantized exactly like engine.py:98-105)."""

    def __init__(self, model_dir, manifest):
        self.path = os.path.join(model_dir, "embeddings.safetensors")
        self.eq = manifest.get("embed_quant") or {}
        if self.eq:
            self.q = safetensors.read_tensor(self.path, "embed.q")
            self.s = safetensors.read_tensor(self.path, "embed.scale")
            self.shape = (self.eq["out"], self.eq["in"])
        else:
            self.t = safetensors.read_tensor(self.path, "embed")
            self.shape = self.t.shape

    def __getitem__(self, idx):
        if not self.eq:
            return np.asarray(self.t[idx], np.float16)
        q = np.asarray(self.q[idx])
        s = np.asarray(self.s[idx], np.float32)
        if self.eq["bits"] == 4:
            q = quant.unpack_int4(q.reshape(1, -1), 1, self.eq["in"]).reshape(-1)
        return (q.astype(np.float32) * np.repeat(s, self.eq["block"], axis=-1)).astype(np.float16)
