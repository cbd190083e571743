"""CPU oracle of Mosaic's block-sparse attention forward — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU reference.
The product (mosaic_b200) never imports it.
"""
