"""TEST INFRASTRUCTURE ONLY -- CPU oracle of the depthwise Conv1D path.

* :mod:`oracle.reference_torch` -- the reference's PyTorch CPU path, restated;
* :mod:`oracle.c_oracle` -- ctypes binding of ``pt_oracle.c`` (FP64 loops);
* ``build_oracle.py`` -- compiles ``liboracle.so`` and, when the reference
  tree is present, the reference's own CUDA kernels into ``_ref/``.

Only tests/, __graft_entry__.smoke() and bench.py (CPU baseline / reference
arm) may use this package; the product package never imports it.
"""
