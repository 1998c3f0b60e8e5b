"""GPU-backed drop-in for androidllm/models/llama.py (``LlamaModel``).

Same constructor and methods as the reference class (``llama.py:57-164``):

* ``layer_forward(x, layer, kv, pos)`` runs one post-norm decoder layer on the
  device.  ``layer`` is the reference's dict of fp16 ``(out, in)`` matrices
  plus ``n_in`` / ``n_post`` (uploaded once per dict and kept resident), or the
  same dict holding shard-format :class:`~androidllm_b200.ops.QuantProj`
  entries (no host dequantization).  ``kv`` is one entry of
  :meth:`prepare_kv`.  ``x`` may hold several rows: rows are consecutive
  positions starting at ``pos`` (a verify pass).
* ``logits(x)`` returns fp16-rounded logits as fp32 ``(rows, vocab)``.
* ``prepare_kv(max_len)`` returns a per-layer list view of one paged fp16
  device cache.
"""
from ..ops import DeviceKV, DeviceModel, QuantProj, default_context, precompute_rope


class KVLayer:
    """``prepare_kv()[li]``: layer ``li`` of a device KV cache."""

    def __init__(self, cache, layer):
        self.cache = cache
        self.layer = layer

    def read(self, pos0, n):
        """(k, v) fp16 (n, kv_heads, head_dim) at positions pos0.. (the reference layout)."""
        return self.cache.read(self.layer, pos0, n)


class KVList(list):
    """List of :class:`KVLayer` sharing one :class:`DeviceKV`."""

    def __init__(self, cache, n_layers):
        super().__init__(KVLayer(cache, i) for i in range(n_layers))
        self.cache = cache


class LlamaModel:
    def __init__(self, canon, embed, final_norm, lm_head=None, device=0, _device_model=None):
        self.canon = canon
        self.hidden = canon["hidden"]
        self.heads = canon["heads"]
        self.kv_heads = canon["kv_heads"]
        self.head_dim = canon["head_dim"]
        self.rope_theta = canon["rope_theta"]
        self.rms_eps = canon["rms_eps"]
        self.embed = embed
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.rope = precompute_rope(self.head_dim, canon["max_len"], self.rope_theta)
        if _device_model is not None:
            self.dm = _device_model
        else:
            self.dm = DeviceModel(default_context(device), canon)
            self.dm.set_embed(embed)
            self.dm.set_final_norm(final_norm)
            if lm_head is not None:
                self.dm.set_head(lm_head if isinstance(lm_head, QuantProj) else QuantProj.from_fp16(lm_head))
            self.dm.finalize()
        self._resident = [None] * canon["layers"]

    @classmethod
    def from_device(cls, dm, embed=None, final_norm=None, lm_head=None):
        m = cls(dm.canon, embed, final_norm, lm_head, _device_model=dm)
        m._resident = list(dm._layer_src)
        return m

    def _ensure_layer(self, li, layer):
        if self._resident[li] is not layer:
            self.dm.set_layer(li, layer)
            self.dm.finalize()
            self._resident[li] = layer

    def layer_forward(self, x, layer, kv, pos):
        """llama.py:71-128: returns fp16 (rows, hidden); mutates kv at pos.."""
        self._ensure_layer(kv.layer, layer)
        return self.dm.layer_forward(kv.layer, kv.cache, x, pos)

    def logits(self, x):
        """llama.py:130-146: fp16-rounded logits as fp32 (rows, vocab)."""
        lg, _ = self.dm.head_logits(x)
        return lg

    def prepare_kv(self, max_len):
        """llama.py:148-164: zeroed per-layer fp16 cache on the device."""
        return KVList(DeviceKV(self.dm, max_len), self.canon["layers"])
