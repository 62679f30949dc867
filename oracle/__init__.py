"""TEST INFRASTRUCTURE — ORACLE ONLY: the CPU restatement of the reference (oracle.c) and the
reference compiled from its own sources (_ref/), used by tests/, __graft_entry__.smoke() and
bench.py's CPU legs as the checker; the product never imports it."""
