"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the b200_cuda kernels.

Importable only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg. The product path (``ace_kernels_b200``) never imports it.
"""
