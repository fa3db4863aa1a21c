"""CPU oracle for the voom_b200 hot path -- TEST INFRASTRUCTURE ONLY.

Restatements of the reference algorithms (plain C compiled with gcc, numpy,
torch-CPU for the expert math) used as the checker by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / --impl reference legs.
The product package (voom_b200) never imports, links or calls anything here.
"""
