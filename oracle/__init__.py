"""CPU oracle for the SR-DiT hot path -- TEST INFRASTRUCTURE ONLY.

A plain numpy / PyTorch-CPU restatement of the reference's algorithms
(AMAP-ML/DreamX-Creator, ``video_refiner/wan/modules/sr_dit/``), each function
citing the reference file:line it follows. It exists to check the CUDA path:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm
may import it. The product package never imports it, and it is never the thing
measured or shipped.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against the
golden vectors in ``tests/golden/``, which ``tests/golden/gen_golden.py``
produced by executing the reference's own Python in this repository's build
container (the reference ships no tests or fixtures of its own).
"""
