"""CPU oracle for the per-layer attention path of NanoSLG.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``) may import
anything here, and only as the checker or the timed reference arm -- never as the thing
measured or shipped.  ``nanoslg_b200`` never imports it.

Each module restates, in plain torch/numpy on the CPU, the reference code it cites
(paths relative to the NanoSLG checkout):

* ``attention``  -- ``ContiguousCacheContext.attend`` with ``_build_causal_mask`` and
  ``_sdpa`` (nanoslg/kv_cache.py:44-56, 192-224, 247-325): the north star's oracle.
* ``rope_norm``  -- ``precompute_rope_frequencies``, ``apply_rotary_emb``, ``RMSNorm``
  (nanoslg/models.py:25-83).
* ``paged_plan`` -- the per-token write targets and the CSR page list of
  ``FlashInferCacheContext`` (nanoslg/kv_cache.py:575-632).
* ``llama``      -- the tiny Llama forward of ``LlamaTP`` at TP=1 (nanoslg/models.py
  :86-172, 246-276) on the contiguous oracle, for greedy-token parity.

Pinning: ``tests/test_oracle_golden.py`` checks every module against the fixtures in
``tests/golden/``, which ``tests/golden/make_golden.py`` recorded by running the
reference itself.
"""
