"""Test-only CPU oracle of the SISA hot path (see ``oracle/sisa_oracle.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this package. The product package ``sisa_b200`` never does.
"""
