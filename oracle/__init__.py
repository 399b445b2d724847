"""CPU oracle for the Z-Image S3-DiT W8A8 forward path (TEST INFRASTRUCTURE ONLY).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path
(``comfyui-zimage-triton_b200``) never imports it and fails loudly when its
CUDA library is missing.

Modules
-------
``ops``    restatement of every op on the path (W8A8 + Hadamard linear,
           weight prep, the six Triton kernels), each function citing the
           reference file:line it follows.
``model``  the S3-DiT block / step composition of the reference's patched
           forwards (``models/patching_comfyui.py``), random-init weights.

Parity pinning: the W8A8 pieces are pinned against the reference's own
``zimage_triton.quantization`` code run on CPU (golden fixtures under
``tests/golden`` made by ``tests/golden/make_golden.py``).  The Triton
kernels cannot run here (the Triton interpreter fails on libdevice and bf16),
so their restatement is pinned only for the fp32 kernels the interpreter can
execute (``swiglu``, ``rope_3d``); the others are parity-unpinned beyond
their line-by-line restatement.
"""
