"""Oracle for mini-flash-attention-b200 -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package. Only tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py use it, and only as the checker or the timed CPU
baseline, never as the computation that is measured or shipped.

Contents:
  attention.py   numpy restatements of the reference algorithm (naive fp32 attention as the
                 reference test computes it, and the blockwise online-softmax recurrence of
                 the reference CuTe kernel, fp16 P rounding included)
  torch_naive.py the reference benchmark's "torch" backend, run on host CPU cores
  build_ref.py   recipe that compiles the reference's own CUDA kernels (unmodified sources)
                 into oracle/_ref/libmfa_ref.so; ref.py loads it (GPU only)
Parity is pinned by tests/golden/ fixtures produced by the reference CuTe kernel itself.
"""
