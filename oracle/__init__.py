"""CPU oracle for the Orca MLP training path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm;
never by the product package `orcaml_b200`.
"""
