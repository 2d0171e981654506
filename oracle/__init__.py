"""CPU oracle for the MiniLM-BERT sentence-embedding path (test infrastructure only).

Nothing in the product path imports this package: only tests, the smoke check and the
CPU-baseline leg of bench.py use it, and only as the checker.
"""
