"""CPU oracle for krunch_b200 — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its CPU-baseline leg and
its `--impl reference` arm) may import this package, and only as the checker
or the timed CPU reference.  The product path (krunch_b200) never imports it.

* kb_oracle.c / coder.py — the range coder of krunch_ac/cpu_reference.py and
  the CDF rule of krunch_ac/cdf.py in plain C (built by oracle/build.py).
* rwkv.py — RWKV-4 forward in numpy fp32 following scripts/rwkv4_step_ref.py
  (stepped) and krunch/batched_rwkv4.py:_att_seq_batched/_ffn_seq_batched
  with KRUNCH_PURE_WKV=1 (packed).

Parity pins: tests/golden/ holds outputs of the reference's own Python code
(cpu_reference.encode, cdf.probs_to_cdf, rwkv4_step_ref.step_one,
batched_rwkv4.forward_batched) produced by tests/golden/make_golden.py; the
oracle is checked against them in tests/test_oracle_golden.py.
"""
