"""Oracle: a CPU restatement of androidllm's speculative-decode path.

THIS PACKAGE IS TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it, and only as the checker or as the
timed CPU baseline.  The product path (``androidllm_b200``) never imports it
and has no CPU fallback.

Every function restates one reference function in plain numpy and cites the
reference file:line it follows (paths are relative to the androidllm project
root).  The arithmetic order and the rounding points are kept identical to the
reference numpy path, because that path is the declared source of truth
(androidllm ``CONTRIBUTING.md:49-52``):

* ``oracle.quant``    - ``androidllm/quant.py`` (block quant, nibble pack,
  dequant).  Pinned by golden vectors produced by the reference itself
  (``tests/golden/make_golden.py``) and by the reference's known-answer pack
  vector (``tests/test_quant.py:39-46`` of the reference).
* ``oracle.llama``    - ``androidllm/models/llama.py`` numpy branch
  (``layer_forward``, ``logits``, ``prepare_kv``).  Pinned by reference
  hidden states and logits on seeded toy models.
* ``oracle.sampling`` - ``androidllm/engine.py:26-45`` sampler and the
  speculative acceptance rules.  The greedy and "target sample == draft
  sample" rules are pinned by reference runs; the min(1, p/q) rejection rule
  has no counterpart in the reference (parity unpinned by the reference; it
  is pinned only against its own definition here).
* ``oracle.engine``   - ``androidllm/engine.py:255-405`` decode loop with
  resident weights.  Pinned by reference greedy / speculative token streams.
* ``oracle.io``       - ``androidllm/safetensors.py`` reader, used to load
  the same shard directories the product loads.
"""
