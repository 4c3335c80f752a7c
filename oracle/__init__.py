"""CPU oracle for the KernelForge hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference's framework-native
baselines (the three ``original.py`` files of zzd1992/KernelForge):

* ``oracle.rmsnorm``  -- RMSNorm forward             (rmsnorm/original.py:9-52)
* ``oracle.sana``     -- SANA LiteLA ``attn_matmul``  (SANA_LinearAttention/original.py:99-117)
* ``oracle.fa_jvp``   -- dense attention / JVP        (flash_attention_jvp/original.py:6-65)

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) may import this package, and only as the checker or the timed CPU
baseline. The product package ``kernelforge_b200`` never imports it: every product entry point
runs the CUDA extension and fails loudly when the extension is missing.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own ``original.py``
code and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks
this oracle against those fixtures.
"""
