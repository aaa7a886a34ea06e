"""krunch_b200 — B200-native (sm_100a) compress/decompress hot path of the
krunch neural text codec.

Python host code over a C-ABI CUDA library (libkrunch_b200.so, declared in
include/krunch_b200.h).  Surfaces that mirror the reference:
  krunch_b200.inference      — engine, .krunch header  (krunch/inference.py)
  krunch_b200.chunking       — chunk sizing / framing  (krunch/chunking.py)
  krunch_b200.cli            — `krunch compress|decompress` (krunch/cli.py)
  krunch_b200.batched_rwkv4  — batched forward         (krunch/batched_rwkv4.py)
  krunch_b200.krunch_ac      — CDF + range coder API   (krunch_ac/)
  krunch_b200.krunch_ac_cuda — the reference extension's function names
"""
__version__ = "0.1.0"
