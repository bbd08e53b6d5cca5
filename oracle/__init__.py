"""CPU oracle for thork_b200 parity tests and CPU baselines (test
infrastructure only; see oracle/oracle.py)."""
