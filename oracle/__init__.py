"""Oracle for the AGILLM4.1 MoE block forward.

This package is TEST INFRASTRUCTURE. It restates, on the CPU (or on any torch
device, for the same-GPU comparison), what the reference's ``MoEFFN.forward``
computes (agillm41.py:4389-4431), so that the CUDA path can be checked against
it. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker or as the timed CPU
baseline. The product path (``agillm41_b200``) never imports it and has no CPU
fallback.

Parity status: the restatement is pinned against golden vectors produced by
the reference module itself (``tests/golden/make_golden.py`` imports the
reference's ``agillm41.py`` and writes ``tests/golden/*.npz``). The reference
ships no test vectors of its own for this path.
"""
