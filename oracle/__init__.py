"""CPU oracle of the NVFP4 Gated DeltaNet path -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
the checker; never by the product (blackwell-kernel-sm_120_b200/).
"""
