"""Oracle package (test infrastructure only): the C restatement of the
reference's per-connection loops and the reference itself compiled from its
own sources. Imported only by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg."""
