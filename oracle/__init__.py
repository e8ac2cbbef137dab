"""Test infrastructure: the CPU oracle for the HBA hot path (see hba_oracle.py).
Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU legs."""
