"""Per-phase timing of the fused decode step (profiling aid).

    python -m krunch_b200.step_trace [B] [--model 169m|1.5b] [--steps N]

Builds the w8a8 model on random weights, runs kb_step_forward for B streams
a few times, then once with kb_step_set_trace: CTA 0 records %globaltimer at
every grid barrier's entry and exit and SM clocks around its first unit of
each tile phase.  Prints the work and barrier time of each phase (first and
last layer), the totals, the tile-phase segments averaged over layers, and
the CUDA-event time per step."""
from __future__ import annotations

import argparse

import numpy as np


def main() -> None:
    import torch
    from . import _native as N
    from .model import RWKVModel
    from .synth import random_weights
    ap = argparse.ArgumentParser()
    ap.add_argument("B", type=int, nargs="?", default=256)
    ap.add_argument("--model", default="169m", choices=["169m", "1.5b"])
    ap.add_argument("--steps", type=int, default=20)
    a = ap.parse_args()
    shape = (12, 768, 3072, 50277) if a.model == "169m" else (24, 2048, 8192, 50277)
    m = RWKVModel(random_weights(*shape, seed=0), wdtype="i8")
    L, B = shape[0], a.B
    tr = torch.zeros(65536, dtype=torch.int64, device="cuda")
    st, ws = m.new_state(B), m.new_step_workspace(B)
    lg, ss = m.new_logits(B, 1), m.new_stats(B, 1)
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    for _ in range(5):
        m.step_forward(tok, st, ws, lg, ss)
    N.call("kb_step_set_trace", tr.data_ptr())
    m.step_forward(tok, st, ws, lg, ss)
    torch.cuda.synchronize()
    N.call("kb_step_set_trace", None)
    t = tr.cpu().numpy().astype(np.int64)
    ent, ex = t[0:512:2], t[1:512:2]
    names = ["embed"] + [f"L{l}:{p}" for l in range(L)
                         for p in ("kvr", "wkv", "o", "ln2", "ffn", "mid", "fv", "ln1")]
    print("phase        work_us  barrier_us")
    tw = tb = 0.0
    e = 1
    while e < len(ent) and ent[e] != 0:
        w = (ent[e] - ex[e - 1]) / 1e3 if e > 1 else 0.0
        b = (ex[e] - ent[e]) / 1e3
        tw, tb = tw + w, tb + b
        if e <= 9 or e > 8 * (L - 1) + 1:
            print(f"{names[e - 1]:12s} {w:7.2f} {b:7.2f}")
        e += 1
    print(f"total work {tw:.1f} us, barriers {tb:.1f} us, span {(ex[e - 1] - ent[1]) / 1e3:.1f} us")
    ti = t[512:512 + 4 * 4 * L].reshape(4 * L, 4)
    acc = np.zeros((4, 4))
    for tp in range(4 * L):
        st0 = t[768 + 2 * tp + 1]
        acc[tp % 4] += np.array([ti[tp, 0] - st0, ti[tp, 1] - ti[tp, 0], ti[tp, 2] - ti[tp, 1],
                                 ti[tp, 3] - ti[tp, 2]]) / 1e3
    print("tile phases (k SM cycles, mean over layers): start->issued issued->landed "
          "landed->MMA done MMA->stored")
    for k, nm in enumerate(["kvr", "o", "ffn", "fv"]):
        print(f"  {nm:4s}", np.round(acc[k] / L, 2))
    t2 = np.zeros((4, 3))
    for tp in range(4 * L):
        st0 = t[768 + 2 * tp + 1]
        x0, x1, x2 = t[1536 + 4 * tp:1536 + 4 * tp + 3]
        t2[tp % 4] += np.array([x0 - st0, x1 - x0, x2 - x1]) / 1e3
    print("tile phase start (k SM cycles): barrier exit->phase entry, ->unit found, ->W issued")
    for k, nm in enumerate(["kvr", "o", "ffn", "fv"]):
        print(f"  {nm:4s}", np.round(t2[k] / L, 2))
    print("row phases (k SM cycles, mean over layers): barrier exit->entry entry->data "
          "data->reduced reduced->end")
    racc = np.zeros((4, 4))
    for l in range(L):
        for j in range(4):
            rp = 1 + 4 * l + j
            r0 = t[1024 + 4 * rp:1024 + 4 * rp + 4]
            ex_clk = t[768 + 8 * l + 2 + 2 * j]
            racc[j] += np.array([r0[0] - ex_clk, r0[1] - r0[0], r0[2] - r0[1], r0[3] - r0[2]]) / 1e3
    for k, nm in enumerate(["wkv", "ln2", "mid", "ln1"]):
        print(f"  {nm:4s}", np.round(racc[k] / L, 2))
    # every CTA's arrival time per barrier: the phase's critical path is the
    # last arrival minus the previous barrier's release
    G = torch.cuda.get_device_properties(0).multi_processor_count
    E = e - 1
    arr = t[2048:2048 + (E + 1) * G].reshape(E + 1, G)
    crit = np.zeros(8)
    med = np.zeros(8)
    rel = np.zeros(8)
    slow = np.zeros(G)
    for ep in range(2, E + 1):
        k = (ep - 2) % 8
        crit[k] += (arr[ep].max() - ex[ep - 1]) / 1e3
        med[k] += (np.median(arr[ep]) - ex[ep - 1]) / 1e3
        rel[k] += (ex[ep] - arr[ep].max()) / 1e3
        slow[arr[ep].argmax()] += 1
    print("per phase (us, summed over layers): critical (last arrival - previous release), "
          "median arrival, release after last arrival")
    for k, nm in enumerate(["kvr", "wkv", "o", "ln2", "ffn", "mid", "fv", "ln1"]):
        print(f"  {nm:4s} crit {crit[k]:7.1f}  median {med[k]:7.1f}  release {rel[k]:6.1f}")
    print(f"  total crit {crit.sum():.1f}  release {rel.sum():.1f}")
    top = np.argsort(-slow)[:8]
    print("slowest CTA counts:", {int(i): int(slow[i]) for i in top})
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        m.step_forward(tok, st, ws, lg, ss)
    e1.record()
    torch.cuda.synchronize()
    print(f"kb_step_forward (layers + head): {e0.elapsed_time(e1) * 1e3 / a.steps:.1f} us/step at B={B}")


if __name__ == "__main__":
    main()
