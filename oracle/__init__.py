"""CPU oracle for the sluice_b200 hot path — TEST INFRASTRUCTURE ONLY.

Nothing in the product package (``sluice_b200``) imports this package. Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` use it, and only as the checker or as the timed CPU baseline,
never as the thing that is measured or shipped.

Contents (each function cites the reference file:line it restates):

* ``slot_policy`` — the router-split gap's SLRU slot cache and expert map
  (``src/sluice/offloader.py`` of kfirtoledo/sluice). Pinned against the
  reference's own ``_router_split_gap`` run on CPU: golden traces under
  ``tests/golden/`` were produced by ``tests/golden/make_golden.py``.
* ``routing`` — router arithmetic (softmax / sigmoid, grouped top-k,
  renormalisation, routed scaling) restated from vLLM 0.22's torch-native
  ``grouped_topk`` / ``select_experts`` (third-party code the reference calls;
  the reference pins vLLM 0.23). Pinned against vLLM's CPU functions run here.
* ``moe`` — ``fused_experts`` semantics through an ``expert_map`` (SwiGLU
  expert MLP, weighted top-k sum, shared experts, fp8 128x128 block-scale
  dequantisation), restated from vLLM's ``cpu_fused_moe_torch`` and
  ``fused_moe.py``. Pinned against vLLM's ``cpu_fused_moe_torch`` run here.

Tie rule: the reference's ``torch.topk(sorted=False)`` leaves the order (and,
at an exact tie on the k-th score, the choice) of the selected experts
implementation-defined. The oracle fixes it: scores descending, expert id
ascending on equal scores. Golden routing vectors avoid k-boundary ties.
"""
