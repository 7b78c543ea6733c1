"""CPU oracle for the streaming AV attention hot path — TEST INFRASTRUCTURE ONLY.

Plain numpy / torch-CPU restatements of the reference's algorithms, each function citing
the reference file:line it follows (paths relative to the reference checkout:
``src/taomate_h3/...`` as ``T/``, ``src/taomate-fl2av/src/digitalhuman_h3/...`` as ``F/``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
legs may import this package, and only as the checker or the timed CPU baseline. The
product path (``h3sa``) never imports it and has no CPU fallback.

Pinning: the golden fixtures under ``tests/golden/`` were produced by running the
reference's own Python code on CPU (``tests/golden/make_golden.py``); the CPU test suite
checks every oracle function against them. The reference ships no golden vectors of its
own for this path.
"""
