"""CPU oracle (test infrastructure only): numpy restatement of the reference's
program semantics. Importable only from tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py."""
