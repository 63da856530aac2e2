"""ORACLE — test infrastructure only.

CPU restatements of the reference's hot-path arithmetic, and wrappers of the
reference's own sources compiled in place (oracle/Makefile -> oracle/_ref/).
Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package. The product path (turboocr_b200) never does.
"""
