"""CPU oracle for the spike-sparse conv path -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker / the timed CPU reference. The product
(sparseflow_b200) never imports it.
"""
