"""CPU oracle for the packed-quant MoE and Q8 KV-cache hot path (TEST INFRASTRUCTURE ONLY).

Nothing in the shipped library imports this package. It is the checker used by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py``.
Every function restates, in plain NumPy, the algorithm of one function of the
reference runtime (AhmadSaeedZaidi/data-synth-tpu, ``kaggle/``) and cites the file
and lines it follows.

Parity pins (see ``tests/test_oracle_golden.py``):

* GGUF decoders are pinned byte-for-byte against the reference's own NumPy decoders
  (``glm53_offload/gguf_quant.py``, ``qwen38_tpu/quant.py``,
  ``packed_q6/reference.py``) and against gguf-py 0.19.0, through fixtures made by
  ``tests/golden/make_golden.py``.
* The packed-Q6 projection oracle is pinned against ``packed_q6/reference.py``'s
  ``projection_reference`` outputs.
* The routed-FFN oracle is pinned against the reference's independent NumPy
  routed-FFN oracle (``qwen38_tpu/routing_validation.py:224-243``) on its own seed.
* The Q8 KV codec is pinned against the reference's ml_dtypes oracle expressions
  (``qwen38_tpu/validation.py:44-52``, ``tests/test_qwen38_kv_gather.py:22-32,88-91``).
* Router top-k has no runnable reference (its JAX path cannot be imported without
  JAX): it is checked against an independent fp64/stable-sort formulation, and that
  part of parity is unpinned.
"""
