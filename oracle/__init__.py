"""CPU oracle for the semantic-ID-constrained beam-search path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm the
reference (amilcodes/RapidTinyRec) runs for one request:

* ``sid_tables``  - ``GpuSidConstraintTables`` (``rapidtinyrec/gpu_constraints.py:17-87``)
  and the released semantic processor (``rapidtinyrec/source/LogitProcessor.py:45-73``);
* ``qwen2_cpu``   - the Qwen2 decoder forward that ``PrefillOnce`` /
  ``PrefillPrefix`` (``shared_prefill.py:27-60``, ``prefix_prefill.py:27-63``) and
  ``folded_sdpa`` (``folded_attention.py:16-31``) drive inside Hugging Face
  ``transformers`` 5.5.0 ``Qwen2ForCausalLM``;
* ``beam_cpu``    - the ``GenerationMixin._beam_search`` loop of ``transformers``
  (third-party; the reference pins 4.55.4, the image holds 5.5.0 whose
  vectorised helpers are the same) plus ``GpuSidConstrainedLogitsProcessor``
  (``gpu_constraints.py:90-101``) and ``compute_transition_scores``.

The oracle is pinned against golden vectors produced by running the reference
itself (``tests/golden/make_golden.py``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it,
and only as the checker / the timed CPU baseline - never as a product path.
"""
