"""TEST INFRASTRUCTURE ONLY: CPU oracles for the fused LNCC loss.

- `oracle.c_oracle`: fp64 C restatement of the reference kernel's semantics (lncc_oracle.c).
- `oracle.torch_port`: a restatement of the reference's PyTorch baseline
  (baselines/torch_lncc.py), used as the timed CPU baseline and as a second parity check.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package, and
only as the checker. The product (fused-lncc_b200/) never does.
"""
