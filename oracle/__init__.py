"""ORACLE — test infrastructure: a CPU/PyTorch restatement of the reference's
training step, against which the B200 kernels are compared. Only tests/,
bench.py's CPU-baseline and reference legs, and __graft_entry__.smoke() may
import it."""
