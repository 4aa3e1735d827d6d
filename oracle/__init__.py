"""CPU oracle for the WKV-7 + ROSA hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (``model.py``, ``scans.py``) and plain C
(``scans_ref.c``), the reference's own PyTorch fp32 CPU path:

* ``RWKV7TimeMix._torch_recurrence``   yufmusicgen/model.py:145-165
* ``ROSAMemory._reference_recurrence`` yufmusicgen/model.py:260-288
* ``YufMusicGen.forward`` / ``.step``  yufmusicgen/model.py:345-431

``wy.py`` restates the WKV-7 chunk summary in the chunked (WY) matrix form, as
the checker for a tensor-core version of the time-parallel scan's first pass.

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The engine in ``yufmusicgen_b200`` never calls into this package
and has no CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree in the build container) on seeded inputs and
writes the fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this oracle against every fixture.
"""
