"""CPU and reference-GPU oracles for the quantized DiT-block linear path.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import this package, and only as
the checker or the timed CPU baseline.  The product (the ``h3_speedkit``
package and its CUDA library) never imports or calls anything here.

* ``oracle.cpu``     -- ctypes binding of the C restatement ``h3_oracle.c``.
* ``oracle.ref_gpu`` -- the reference's own CUDA kernels compiled into
  ``oracle/_ref`` (see ``oracle/build.py``), the bit-exact GPU checker.
* ``oracle.chain``   -- the DiT block chain composed from ``oracle.cpu``.
"""
