"""CPU oracle for the MiracleReasoning token loop — TEST INFRASTRUCTURE ONLY.

This package is the checker the CUDA product is compared against: a plain-C
restatement of the reference kernels (``kernels.c``), a host build of the
reference's own ``kernels.cl`` (``ref_host.cpp`` -> ``_ref/``), a host backend
with the reference backend's method surface (``host_backend``) and a
restatement of the reference token loop (``reference_model``).  Only the test
suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it; the product package never does, and never falls back to it.
"""
