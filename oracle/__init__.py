"""CPU oracle of the MOSS-Image int8 hot path - TEST INFRASTRUCTURE ONLY.

Restates the reference algorithms (``training/quantization.py``,
``training/quant_kernels.py``, ``training/activation_offload.py``) in plain C
(``w8_oracle.c``) and numpy (``oracle.py``) so the CUDA path can be checked against them.
It is pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``). Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it; the product package never does.
"""
