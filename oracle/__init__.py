"""
ORACLE — test infrastructure, not product code. CPU restatements of the reference's rasterization hot path (oracle.c, via cpu.py), its
quantization (quant.py) and rate term (rate.py), used only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
checker. Nothing in the igs_b200 product imports it.
"""
