"""Test-only CPU oracle for the TurboQuant KV-cache path (see tq_oracle.py)."""
