"""CPU oracle for the packed mixed-batch forward: TEST INFRASTRUCTURE ONLY.

This package restates, in plain Python and PyTorch-on-CPU, the algorithm of
Helios's packed tick (the reference project, sidmanale643/helios) so the CUDA
path in ``helios_b200`` can be checked against it. It is a checker, never the
thing measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path (``helios_b200``) never imports it and raises when its CUDA
library is missing.

Parity pin: ``tests/golden/make_golden.py`` imports the reference itself (in the
build container, where its sources are present) and writes golden vectors to
``tests/golden/``; ``tests/test_oracle_golden.py`` checks every function here
against them. The fixtures cover the reference's own known-answer metadata
(``tests/test_paged_attention.py:97-118, :262-263``), the page-boundary case
(``:59-74``), BASELINE config 1 (tiny fp32 Qwen3, logits + 16 greedy steps) and a
bf16 mixed tick at the Qwen3-4B head shape.

Modules:
    metadata   -- tick packing (``paged_cache.py:221-270``, ``:418-494``)
    numerics   -- RMSNorm and RoPE (``layers.py:30-72``)
    attention  -- causal paged GQA attention (``paged_cache.py:378-414``, ``:521-546``)
    model      -- Qwen3 weights and packed forward (``model.py:13-110``, ``layers.py:13-232``)
    sampler    -- greedy / temperature / top-p rule (``decode.py:457-473``)
"""
