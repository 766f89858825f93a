"""TEST INFRASTRUCTURE ONLY: CPU checkers for the lmpb kernels.

``oracle.port``  — numpy front-end of liblamp3_oracle.so, the plain-C
                   restatement of the reference Lamp3 CPU kernels.
``oracle.ref``   — the reference's own CPU core (built from its sources into
                   _ref/liblamp3_ref.so) through a small C harness.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package; the product never does.
"""
