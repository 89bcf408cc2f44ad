"""Test infrastructure: the CPU oracle for the Sdpa / SdpaGrad hot path.

Only tests/, __graft_entry__.smoke() and bench.py (its reference arm and
cpu_baseline leg) may use this package -- as the checker, never as the thing
measured or shipped.

  oracle.cpu   -- ctypes driver of sdpa_oracle.c, a C restatement of the
                  reference GPU algorithm (liboracle.so)
  oracle.ref   -- ctypes driver of the reference's own op sources built
                  unmodified against tf_shim/ (oracle/_ref/*.so)
  oracle.dense -- float64 dense attention with the reference's dropout mask
"""
