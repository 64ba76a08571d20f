"""CPU oracle for the routed micro-expert channel mixer.

TEST INFRASTRUCTURE ONLY.  Nothing in ``spalmer_b200`` imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or as
the timed CPU restatement -- never as the measured or shipped GPU path.

It restates the reference algorithm (``mESmaC/spalmer``, Python/PyTorch) in
numpy plus one small C++ file:

* ``bf16``      -- bfloat16 storage/rounding helpers (round-to-nearest-even,
                  canonical NaN), matching ``c10::BFloat16``.
* ``topk``      -- the CPU top-k tie order: ``std::nth_element`` (or
                  ``std::partial_sort`` when ``k*64 <= n``) followed by
                  ``std::sort`` of the first ``k-1`` entries, as PyTorch's
                  ``ATen/native/TopKImpl.h:44-89`` does for the reference's
                  ``scores.topk(k, largest=False)`` (``experts/router.py:92``).
* ``mixer_ref`` -- the full layer forward with the reference's BF16 rounding
                  points (``experts/mixer.py:145-241``).

Parity pins: ``tests/golden/`` holds fixtures produced by importing the
reference itself (``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this oracle against them before any GPU test trusts it.
"""
