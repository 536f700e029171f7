"""CPU oracle of the GGUF dequant + matvec path: TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference legs of ``bench.py`` as the checker; never by ``flatrun_b200``.
``_ref/`` (built by ``make -C oracle``) holds the reference's own native CPU
kernels compiled from its sources.
"""
