"""Test-only checkers: the C restatement (liboracle.so) and the compiled reference (_ref/libclm_ref.so).

Only tests/, the smoke check and bench.py's CPU-baseline / reference legs import this package.  The
product package (clusterlm_b200) never does.
"""
