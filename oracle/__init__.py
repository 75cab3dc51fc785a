"""CPU oracle for the nxv_* hot path -- TEST INFRASTRUCTURE ONLY.

Importable only by tests/, __graft_entry__.smoke() and the CPU-baseline leg
of bench.py.  The product (nx_vulkan_b200) never imports it.
"""
