"""CPU oracle for the triton-llm decode hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic (ziliangpeng/triton-llm),
each function citing the reference file:line it follows. It is the checker
for the CUDA path, never part of it: only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg (``cpu_baseline`` / ``--impl reference``)
may import it. The product package (``triton-llm_b200/``) never does.

Pinning: ``tests/golden/`` holds vectors produced by running the reference
itself (its Triton kernels under ``TRITON_INTERPRET=1`` with a host-memory
allocator, see ``tests/golden/gen_golden.py``); ``tests/test_oracle.py``
checks this restatement against them.
"""

from . import ops, models  # noqa: F401
