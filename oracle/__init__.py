"""CPU oracle for tinyserver_b200's parity tests (test infrastructure only).

Nothing in the ``tinyserver_b200`` package imports this package.
"""
