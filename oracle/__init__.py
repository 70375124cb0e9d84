"""PARITY ORACLE (test infrastructure only).

CPU restatement of chomik-grad's reference ``cpu`` compiler used to check the
cuda-b200 kernels.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import it; the plugin itself never does.
"""
