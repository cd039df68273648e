"""CPU oracle for the mouse-core attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of the reference
(micahr234/mouse-core v0.4.0) for the path rebuilt by ``mouse_core_b200``:

* ``oracle.policy``    grow-then-rebuild policy, packing index maps and
                       segment position ids (integer work, bit-exact).
* ``oracle.attention`` paged/cached decode attention and packed
                       segment-causal attention forward + backward (float64).
* ``oracle.decoder``   the decoder-layer loop of ``FlexDecodeSession.forward``
                       and ``flex_packed_forward`` (Qwen3 / Llama layouts).

It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it. The product package
``mouse_core_b200`` never imports it and has no CPU fallback.

Pinning: every function here is checked by ``tests/test_oracle_golden.py``
against fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by importing and running the reference itself, and against the
known-answer vectors of the reference's own tests.
"""
