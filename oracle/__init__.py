"""CPU oracle for the sparse-MoE expert FFN path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the seruva19/mirai routed
expert path so that the CUDA kernels in ``mirai_b200`` can be checked against
it.  It is imported only by ``tests/``, by ``__graft_entry__.smoke()`` (as the
checker) and by ``bench.py`` (the ``cpu_baseline`` leg and the
``--impl reference`` arm).  The product path (``mirai_b200``) never imports,
calls or links anything in here; it fails loudly when its CUDA library is
missing instead of falling back to the CPU.

Parity status:
  * routing (top-k sets), dispatch plan, permute/combine and INT8 quantisation
    are pinned against golden vectors produced by the reference itself
    (``tests/golden/make_golden.py`` imports the reference and runs it);
  * the routed expert forward/dX semantics are pinned the same way, with
    weights fed through the reference's ``bind_physical_weight_provider`` seam;
  * NF4 bytes are *unpinned* at the bitsandbytes boundary: bitsandbytes 0.49.2
    (the reference's NF4 dependency, ``pyproject.toml:46``) is not installed and
    its source is not part of the reference tree.  ``oracle.quant`` restates the
    published NF4 (QLoRA) and dynamic-tree (8-bit optimizers) constructions and
    the buffer layout the reference stores; the kernels read the code tables
    from the buffers, so decoding is exact given the buffers.
"""
