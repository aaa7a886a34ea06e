"""Benchmark of the krunch compress hot path.

Workload (per GPU): RWKV-4-169M (12 x 768, FFN 3072, vocab 50277), fp16
random-init weights (seed 0); B = 64 chunks x T = 4096 token ids drawn
i.i.d. Zipf(1.1) over the vocabulary through a seeded permutation (seed =
rank); full packed forward, head logits, 16-bit CDF, GPU range encode.  One
step = compressing that whole batch.  Synthetic data: no corpus, tokenizer
file or pretrained weights exist in this environment.

value : MB/s of input with the inputs resident in HBM (bytes = tokens x
        bytes_per_token, 1 byte per token: the byte-level tokenizer this build
        ships); whole job over all ranks, time = max over ranks (CUDA events).
e2e   : the same through the public batch API (Codec.compress_batches): per
        step the token ids go in from pinned host memory and the bitstreams
        come back to the host; the API prepares and enqueues batch i+1 while
        batch i runs.  e2e.sequential: one plan at a time (upload, run, fetch).
roofline : the dominant kernel family (the layer GEMMs), FLOPs / event time.
cpu_baseline : the CPU oracle port (numpy fp32 forward + C CDF + C coder)
        on a bounded sample, rank 0 at N = 1.

--impl reference runs that CPU port (the reference's own path is Python +
CUDA that needs the absent `rwkv` package, so its CPU restatement stands in)
on rank 0 with all host threads.

Multi-GPU: one process per GPU (torchrun); each rank compresses its own 64
chunks (weak scaling, no data-path collective).

stress_1b5 : BASELINE configs[4] (RWKV-4 1.5B architecture): bf16 compress
        B=512 x T=2048 and w8a8 decompress B=512 x 1024 steps per GPU.
box   : BASELINE configs[3] on a bounded slice (--box-chunks 1 MiB log-line
        chunks per GPU): chunk i on rank i mod G through the engine's batch
        API with the w8a8 model, then the NCCL length all-gather + payload
        gather and the rank-0 stitch; reports the collective's share.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "compress MB/s of input (RWKV-4-169M, 16-bit CDF, byte-exact)"
BYTES_PER_TOKEN = 1.0
SHAPES = {"169m": dict(n_layer=12, n_embd=768, n_ffn=3072, n_vocab=50277),
          # the larger-model stress case
          "1.5b": dict(n_layer=24, n_embd=2048, n_ffn=8192, n_vocab=50277)}
SHAPE = SHAPES["169m"]

# DRAM bytes (read + write) per launch of the dominant GEMM, from one ncu
# capture of the ffn-key GEMM (k_gemm_tc<3,256,0>, M = 16384 rows: 30.0 MB
# read + 50.0 MB written) scaled by 4 to the bench's 65536-row launches
# (traffic grows with M).
GEMM_TRAFFIC = 4 * (29.979136e6 + 50.308352e6)
GEMM_TRAFFIC_NOTE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the ffn-key GEMM at "
                     "M=16384 x4 = per 65536-row launch; algorithmic 4 x (25.2 + 4.7 + 100.7) MB")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v
                          and "Not" not in v})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def cpu_port_compress(n_chunks: int, n_tok: int, bits: int, threads: int):
    """The CPU oracle pipeline on n_chunks x n_tok Zipf tokens; returns (seconds, tokens)."""
    import torch  # noqa: F401  (numpy BLAS threads follow the process env)
    from krunch_b200.synth import random_weights, zipf_tokens
    from oracle import coder, rwkv
    w = random_weights(**SHAPE, seed=0)
    toks = zipf_tokens((n_chunks, n_tok), seed=0)
    inp = np.concatenate([np.zeros((n_chunks, 1), np.int32), toks[:, :-1]], axis=1)
    t0 = time.perf_counter()
    lg, _ = rwkv.forward(w, inp)
    lh = coder.lohi_from_logits(lg.reshape(-1, lg.shape[-1]).astype(np.float16),
                                toks.reshape(-1), bits, threads=threads)
    lh = lh.reshape(n_chunks, n_tok, 2)
    total = sum(len(coder.encode_lohi(lh[b], bits)) for b in range(n_chunks))
    dt = time.perf_counter() - t0
    return dt, n_chunks * n_tok, total


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    for _ in range(args.warmup if args.warmup < 1 else 1):
        cpu_port_compress(1, 16, args.cdf_bits, threads)
    times, toks = [], 0
    for _ in range(args.steps):
        dt, n, _ = cpu_port_compress(args.ref_chunks, args.ref_tokens, args.cdf_bits, threads)
        times.append(dt)
        toks = n
    sec = float(np.mean(times))
    v = toks * BYTES_PER_TOKEN / sec / 1e6
    sample = f"{args.ref_chunks} chunks x {args.ref_tokens} tokens of the config workload per step"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "MB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config(args),
        "cpu_baseline": {"value": v, "unit": "MB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "MB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def bench_decompress(args, rank, world, stream, max_over_ranks, barrier):
    """w8a8 RWKV-4-169M, B streams decoded in lock-step, one token
    per stream per step (fused step kernel + head + decode kernel per step,
    replayed as a CUDA graph).  Streams are compressed first by the packed
    path of the same int8 model; the decoded tokens must equal the input."""
    import torch
    from krunch_b200.codec import Codec, DecompressPlan
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import random_weights, zipf_tokens
    Bd, Td = args.dec_B, args.dec_T
    model = RWKVModel(random_weights(**SHAPE, seed=0), device=stream.device, wdtype="i8")
    codec = Codec(model, cdf_bits=args.cdf_bits)
    seqs = list(zipf_tokens((Bd, Td), seed=100 + rank))
    streams = codec.compress_tokens(seqs)
    lens = [len(s) for s in streams]
    dp = DecompressPlan(codec, lens, [Td] * Bd)
    dp.upload(streams)
    dp.run()  # warm-up, graph capture
    torch.cuda.synchronize()
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(stream.device.index) as clk:
        d0.record(stream)
        dp.run()
        d1.record(stream)
        torch.cuda.synchronize()
    barrier()
    dms = max_over_ranks(d0.elapsed_time(d1))
    ok = all(np.array_equal(a, b) for a, b in zip(dp.fetch(), seqs))
    # end to end through the plan API: bitstreams from pinned host memory in,
    # tokens out, inside the timed region
    del dp
    warm = DecompressPlan(codec, lens, [Td] * Bd)  # allocator warm-up, untimed
    del warm
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dp2 = DecompressPlan(codec, lens, [Td] * Bd)
    dp2.upload(streams)
    dp2.run()
    out = dp2.fetch()
    e1.record(stream)
    torch.cuda.synchronize()
    ems = max_over_ranks(e0.elapsed_time(e1))
    ok = ok and all(np.array_equal(a, b) for a, b in zip(out, seqs))
    # the same decode at the engine's default batch (compute_decompress_batch:
    # the reference's formula, SMs x 8 = 1184 streams on B200), fewer steps
    from krunch_b200.codec import compute_decompress_batch
    Bp, Tp = compute_decompress_batch(-1, stream.device), args.dec_default_T
    seqs_p = list(zipf_tokens((Bp, Tp), seed=500 + rank))
    streams_p = codec.compress_tokens(seqs_p)
    dpp = DecompressPlan(codec, [len(x) for x in streams_p], [Tp] * Bp)
    dpp.upload(streams_p)
    dpp.run()  # warm-up, graph capture
    dpp2 = DecompressPlan(codec, [len(x) for x in streams_p], [Tp] * Bp)
    dpp2.upload(streams_p)
    torch.cuda.synchronize()
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    dpp2.run()
    p1.record(stream)
    torch.cuda.synchronize()
    pms = max_over_ranks(p0.elapsed_time(p1))
    ok_p = all(np.array_equal(a, b) for a, b in zip(dpp2.fetch(), seqs_p))
    at_default = {"streams": Bp, "steps": Tp, "us_per_step": pms * 1e3 / Tp,
                  "value": Bp * Tp * world * BYTES_PER_TOKEN / (pms / 1e3) / 1e6, "unit": "MB/s",
                  "byte_exact": bool(ok_p)}
    del dpp, dpp2
    sp = SHAPE
    C, F, L, V = sp["n_embd"], sp["n_ffn"], sp["n_layer"], sp["n_vocab"]
    w_bytes = L * (5 * C * C + 2 * C * F) + C * V          # int8 weights read per step
    s_bytes = 2 * L * 5 * Bd * C * 4                        # fp32 state read + written
    us = dms * 1e3 / Td
    pk, pk_kind = peaks()
    ach = (w_bytes + s_bytes) / (us * 1e-6) / 1e9
    tok = Bd * Td * world
    return {"workload": f"configs[2] decompress: w8a8 RWKV-4-169M, B={Bd} x {Td} steps per GPU, "
                        "fp32 state, CUDA graph of (fused step, head, decode) per step",
            "value": tok * BYTES_PER_TOKEN / (dms / 1e3) / 1e6, "unit": "MB/s",
            "us_per_step": us, "byte_exact": bool(ok), "gpu_launches_per_step": 3,
            "bits_per_token": 8.0 * sum(lens) / (Bd * Td),
            "roofline": {"bound": "hbm", "achieved": ach, "unit": "GB/s", "peak": pk["hbm_gbs"],
                         "peak_kind": pk_kind, "frac": ach / pk["hbm_gbs"],
                         "algorithmic_bytes_per_step": w_bytes + s_bytes},
            "e2e": {"value": tok * BYTES_PER_TOKEN / (ems / 1e3) / 1e6, "unit": "MB/s",
                    "h2d_bytes_per_step": dp2.h2d_bytes, "d2h_bytes_per_step": dp2.d2h_bytes},
            "at_default_batch": at_default,
            "clocks": clk.summary()}


def bench_box(args, rank, world, dev, max_over_ranks, barrier):
    """configs[3] on a bounded slice: seeded log lines cut into 1 MiB
    UTF-8-safe chunks (reference chunking.py:115-138), chunk i compressed on
    rank i mod G by the w8a8 model through the engine's public batch API,
    then the length all-gather + payload gather over NCCL and the rank-0
    stitch into one .krunch blob (krunch_b200.distributed, the path of
    `krunch compress` under torchrun).  Timed: host text -> stitched blob,
    synchronised device and barrier on both sides, max over ranks; the
    collective is timed on its own as well."""
    import zlib

    import torch
    from krunch_b200 import chunking
    from krunch_b200 import distributed as kd
    from krunch_b200 import inference
    from krunch_b200.inference import CodecConfig, decode_header, encode_header
    from krunch_b200.synth import log_lines
    from krunch_b200.tokenizer import ByteTokenizer
    cb = args.box_chunk_bytes
    raw = log_lines(args.box_chunks * world * cb, seed=4)
    eng = inference.engine
    eng.load(CodecConfig(family="169m", cdf_bits=args.cdf_bits, wdtype="i8"), ByteTokenizer(), dev)
    # warm-up, untimed: model, plans, graphs, and the gather's NCCL
    # peer-to-peer connections (set up on first use)
    kd.gather_payloads(eng.compress_chunks_batched([raw[:4096]] * 2), 2 * world)
    chunks = chunking.split(raw, chunk_size=cb)
    mine = [chunks[i] for i in kd.shard(len(chunks), rank, world)]
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    local = eng.compress_chunks_batched(mine)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    payloads = kd.gather_payloads(local, len(chunks))
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    blob = None
    if payloads is not None:
        crc = zlib.crc32(raw) & 0xFFFFFFFF
        blob = encode_header(len(raw), len(chunks), crc) + b"".join(
            chunking.pack_entries(chunks, payloads))
    t3 = time.perf_counter()
    barrier()
    total_s = max_over_ranks(t3 - t0)
    gather_s = max_over_ranks(t2 - t1)
    compress_s = max_over_ranks(t1 - t0)
    ok = None
    if blob is not None:
        hdr = decode_header(blob)
        ents = chunking.parse_entries(blob[inference.HEADER_SIZE:], hdr["n_chunks"])
        ok = (hdr["original_len"] == len(raw) and hdr["flags"] == 0 and
              [ol for ol, _ in ents] == [len(c) for c in chunks])
    return {"workload": f"configs[3] slice: {len(chunks)} log-line chunks of {cb >> 10} KiB "
                        f"({args.box_chunks} per GPU), w8a8 RWKV-4-169M, round-robin over "
                        f"{world} GPU(s), NCCL length all-gather + payload gather, rank-0 stitch",
            "value": len(raw) / total_s / 1e6, "unit": "MB/s", "input_bytes": len(raw),
            "blob_bytes": None if blob is None else len(blob),
            "bits_per_byte": None if blob is None else 8.0 * len(blob) / len(raw),
            "s_total": total_s, "s_compress": compress_s, "s_gather": gather_s,
            "collective_share": gather_s / total_s, "blob_ok": ok,
            "timing": "host perf_counter around device-synchronised steps, max over ranks"}


def bench_stress(args, rank, world, dev, max_over_ranks, barrier):
    """the RWKV-4 1.5B architecture (24 x 2048, FFN 8192),
    random-init weights drawn on the device (synth.random_weights_device).
    Compress: bf16 weights, B chunks x T tokens, W warm-up steps then K timed
    steps (CUDA events).  Decompress: w8a8 weights, B streams stepped for
    dec_T steps (per-op kernels: the fused step is sized for 169M), streams
    compressed first by the same model; byte-exactness checked."""
    import torch
    from krunch_b200.codec import Codec, CompressPlan, DecompressPlan
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import random_weights_device, zipf_tokens
    sh = SHAPES["1.5b"]
    C, F, L, V = sh["n_embd"], sh["n_ffn"], sh["n_layer"], sh["n_vocab"]
    w = random_weights_device(**sh, seed=0, device=dev)
    pk, pk_kind = peaks()
    out = {"workload": f"configs[4] 1.5B stress: compress bf16 B={args.stress_B} x "
                       f"T={args.stress_T}, decompress w8a8 B={args.stress_B} x "
                       f"{args.stress_dec_T} steps, per GPU"}
    # ---- compress, bf16 ----
    model = RWKVModel(w, device=dev, wdtype="bf16")
    codec = Codec(model, cdf_bits=args.cdf_bits)
    B, T = args.stress_B, args.stress_T
    seqs = list(zipf_tokens((B, T), seed=200 + rank))
    plan = CompressPlan(codec, [T] * B)
    plan.upload(seqs)
    for _ in range(args.warmup):
        plan.run()
    torch.cuda.synchronize()
    barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.stress_steps):
            plan.run()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.stress_steps)
    flop_tok = 2.0 * (L * (5 * C * C + 2 * C * F) + C * V)
    tf = B * T * flop_tok / (ms / 1e3) / 1e12
    out["compress"] = {"value": B * T * world * BYTES_PER_TOKEN / (ms / 1e3) / 1e6, "unit": "MB/s",
                       "ms_per_step": ms, "steps": args.stress_steps, "warmup": args.warmup,
                       "dtype": "bf16", "achieved_tflops": tf,
                       "frac_of_sustained_bf16": tf / pk["bf16_tflops_sustained"],
                       "peak_kind": pk_kind, "clocks": clk.summary()}
    del plan, codec, model
    torch.cuda.empty_cache()
    # ---- decompress, w8a8 ----
    model = RWKVModel(w, device=dev, wdtype="i8")
    del w
    codec = Codec(model, cdf_bits=args.cdf_bits)
    Td = args.stress_dec_T
    seqs = list(zipf_tokens((B, Td), seed=300 + rank))
    streams = codec.compress_tokens(seqs)
    lens = [len(s) for s in streams]
    dp = DecompressPlan(codec, lens, [Td] * B)
    dp.upload(streams)
    dp.run()  # warm-up, graph capture
    torch.cuda.synchronize()
    dp2 = DecompressPlan(codec, lens, [Td] * B)
    dp2.upload(streams)
    torch.cuda.synchronize()
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    dp2.run()
    d1.record(stream)
    torch.cuda.synchronize()
    dms = max_over_ranks(d0.elapsed_time(d1))
    ok = all(np.array_equal(a, b) for a, b in zip(dp2.fetch(), seqs))
    w_bytes = L * (5 * C * C + 2 * C * F) + C * V
    us = dms * 1e3 / Td
    ach = (w_bytes + 2 * L * 5 * B * C * 4) / (us * 1e-6) / 1e9
    out["decompress"] = {"value": B * Td * world * BYTES_PER_TOKEN / (dms / 1e3) / 1e6,
                         "unit": "MB/s", "us_per_step": us, "byte_exact": bool(ok),
                         "hbm_frac": ach / pk["hbm_gbs"], "peak_kind": pk_kind}
    del dp, dp2, codec, model
    torch.cuda.empty_cache()
    return out


def config(args):
    name = "RWKV-4-169M" if args.model == "169m" else "RWKV-4 1.5B architecture"
    wl = ("configs[1] compress, packed forward, 1 GPU per rank" if args.model == "169m"
          else "configs[4] compress (1.5B stress), packed forward, 1 GPU per rank")
    return {"workload": wl,
            "model": f"{name} random-init {dict(i8='w8a8 int8', bf16='bf16', f16='fp16')[args.wdtype]}",
            "chunks_per_gpu": args.B,
            "tokens_per_chunk": args.T, "cdf_bits": args.cdf_bits,
            "bytes_per_token": BYTES_PER_TOKEN, "token_dist": "Zipf(1.1) via seeded permutation",
            "global_batch": args.B * args.gpus, "seq_len": args.T,
            "parallelism": f"chunk-replica x{args.gpus}",
            "l2": "inputs larger than L2 (fp16 logits window >> 126 MB)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--B", type=int, default=64)
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--cdf-bits", type=int, default=16)
    ap.add_argument("--ref-chunks", type=int, default=4)
    ap.add_argument("--ref-tokens", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", default="169m", choices=sorted(SHAPES))
    ap.add_argument("--wdtype", default="f16", choices=["f16", "bf16", "i8"],
                    help="weights of the compress line (the decompress line is always w8a8)")
    ap.add_argument("--no-decompress", action="store_true",
                    help="skip the configs[2] decompress line (w8a8, B=256 x 2048 steps)")
    ap.add_argument("--dec-B", type=int, default=256)
    ap.add_argument("--dec-T", type=int, default=2048)
    ap.add_argument("--dec-default-T", type=int, default=256,
                    help="steps of the decode at the engine's default batch")
    ap.add_argument("--no-box", action="store_true",
                    help="skip the configs[3] slice (log lines, 1 MiB chunks, NCCL stitch)")
    ap.add_argument("--box-chunks", type=int, default=8, help="1 MiB chunks per GPU")
    ap.add_argument("--box-chunk-bytes", type=int, default=1 << 20)
    ap.add_argument("--no-stress", action="store_true",
                    help="skip the configs[4] 1.5B stress lines")
    ap.add_argument("--stress-B", type=int, default=512)
    ap.add_argument("--stress-T", type=int, default=2048)
    ap.add_argument("--stress-steps", type=int, default=1)
    ap.add_argument("--stress-dec-T", type=int, default=1024)
    args = ap.parse_args()
    global SHAPE
    SHAPE = SHAPES[args.model]
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    from krunch_b200 import _native as N
    from krunch_b200 import distributed as kd
    from krunch_b200.codec import Codec, CompressPlan
    from krunch_b200.model import RWKVModel
    from krunch_b200.synth import random_weights, zipf_tokens

    kd.init_from_env()
    rank, world = kd.rank(), kd.world()
    args.gpus = world
    dev = torch.device("cuda", kd.local_rank() % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    w = random_weights(**SHAPE, seed=0)
    model = RWKVModel(w, device=dev, wdtype=args.wdtype)
    del w
    codec = Codec(model, cdf_bits=args.cdf_bits)
    toks = zipf_tokens((args.B, args.T), seed=rank)
    seqs = list(toks)
    plan = CompressPlan(codec, [args.T] * args.B)
    plan.upload(seqs)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing ------------------------------------------
    for _ in range(args.warmup):
        plan.run()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            plan.run()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    # the same K steps again with every launch bracketed by CUDA events (the
    # per-kernel durations of the roofline); a separate pass because events
    # between launches keep a kernel from starting during the previous one's
    # tail (programmatic dependent launch), which the headline pass allows
    N.profile_begin()
    for _ in range(args.steps):
        plan.run()
    torch.cuda.synchronize()
    prof = N.profile_end()
    streams = plan.fetch()
    comp_bytes = sum(len(s) for s in streams)
    tokens_all = args.B * args.T * world
    value = tokens_all * BYTES_PER_TOKEN / (ms / 1e3) / 1e6
    launches = int(sum(v[1] for v in prof.values())) // args.steps

    # ---- roofline of the dominant kernel family -----------------------------
    pk, pk_kind = peaks()
    if args.wdtype == "i8":  # dense int8 runs at twice the bf16 rate on B200
        pk = dict(pk, bf16_tflops_sustained=2 * pk["bf16_tflops_sustained"])
        pk_kind += ", int8 peak = 2 x bf16"
    dom = max(("gemm", "head", "cdf", "wkv", "ln_mix"), key=lambda k: prof[k][0])
    kern = {}
    for k, (kms, n, work) in prof.items():
        if n == 0:
            continue
        if k in ("gemm", "head"):
            ach = work / (kms / 1e3) / 1e12
            kern[k] = {"ms_per_step": kms / args.steps, "launches_per_step": n // args.steps,
                       "achieved": ach, "unit": "TFLOP/s",
                       "frac": ach / pk["bf16_tflops_sustained"]}
        else:
            ach = work / (kms / 1e3) / 1e9
            kern[k] = {"ms_per_step": kms / args.steps, "launches_per_step": n // args.steps,
                       "achieved": ach, "unit": "GB/s", "frac": ach / pk["hbm_gbs"]}
    d = kern[dom]
    roofline = {"kernel": dom, "bound": "tensor" if d["unit"] == "TFLOP/s" else "hbm",
                "achieved": d["achieved"], "unit": d["unit"],
                "peak": pk["bf16_tflops_sustained"] if d["unit"] == "TFLOP/s" else pk["hbm_gbs"],
                "peak_kind": f"{pk_kind} (bf16 sustained / HBM copy)", "frac": d["frac"],
                "traffic": GEMM_TRAFFIC if dom == "gemm" and args.model == "169m" else None,
                "traffic_note": GEMM_TRAFFIC_NOTE if dom == "gemm" and args.model == "169m" else None,
                "per_family": kern}

    # ---- end-to-end through the public API ---------------------------------
    # a plan per step, as a caller compressing batch after batch would; the
    # device-resident plan is released first and one untimed plan warms the
    # allocator, so the timed steps reuse cached device and pinned blocks
    del plan
    p2 = CompressPlan(codec, [args.T] * args.B)
    p2.upload(seqs)
    p2.run()
    p2.fetch()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(max(1, args.steps)):
        p2 = None
        p2 = CompressPlan(codec, [args.T] * args.B)
        p2.upload(seqs)
        p2.run()
        out2 = p2.fetch()
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e2.elapsed_time(e3) / max(1, args.steps))
    wall_ms = (time.perf_counter() - t0) * 1e3 / max(1, args.steps)
    assert out2 == streams, "compress is not deterministic across runs"
    # the same K batches through the pipelined batch API (Codec.compress_batches):
    # every batch still goes host -> device -> host through pinned memory, but
    # batch i+1 is planned, uploaded and enqueued while batch i runs; one
    # untimed pass warms the allocators for two plans alive at once
    for _ in codec.compress_batches([seqs] * 2):
        pass
    torch.cuda.synchronize()
    barrier()
    t1 = time.perf_counter()
    e4 = torch.cuda.Event(enable_timing=True)
    e5 = torch.cuda.Event(enable_timing=True)
    e4.record(stream)
    outs = list(codec.compress_batches([seqs] * max(1, args.steps)))
    e5.record(stream)
    torch.cuda.synchronize()
    pipe_ms = max_over_ranks(e4.elapsed_time(e5) / max(1, args.steps))
    pipe_wall_ms = (time.perf_counter() - t1) * 1e3 / max(1, args.steps)
    assert all(o == streams for o in outs), "pipelined compress differs"
    e2e = {"value": tokens_all * BYTES_PER_TOKEN / (pipe_ms / 1e3) / 1e6, "unit": "MB/s",
           "h2d_bytes_per_step": p2.h2d_bytes, "d2h_bytes_per_step": p2.d2h_bytes,
           "api": "Codec.compress_batches (pipelined: batch i+1 prepared while batch i runs)",
           "wall_ms_per_step": pipe_wall_ms,
           "sequential": {"value": tokens_all * BYTES_PER_TOKEN / (e2e_ms / 1e3) / 1e6,
                          "unit": "MB/s", "api": "CompressPlan upload/run/fetch per batch",
                          "wall_ms_per_step": wall_ms}}

    extra = {}
    if not args.no_decompress:
        extra["decompress"] = bench_decompress(args, rank, world, stream, max_over_ranks, barrier)

    if not args.no_box:
        extra["box"] = bench_box(args, rank, world, dev, max_over_ranks, barrier)
    if not args.no_stress and args.model == "169m":
        extra["stress_1b5"] = bench_stress(args, rank, world, dev, max_over_ranks, barrier)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        dt, n, _ = cpu_port_compress(args.ref_chunks, args.ref_tokens, args.cdf_bits, threads)
        cpu = {"value": n * BYTES_PER_TOKEN / dt / 1e6, "unit": "MB/s", "cores": threads,
               "kind": "port",
               "sample": f"{args.ref_chunks} chunks x {args.ref_tokens} tokens, {dt:.1f} s"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "MB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.wdtype,
                "data": "synthetic (Zipf token ids, random-init weights)",
                "config": config(args), "tokens_per_s": tokens_all / (ms / 1e3),
                "bits_per_token": 8.0 * comp_bytes / (args.B * args.T),
                "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu,
                "e2e": e2e, "clocks": clk.summary(), **extra}
        print(json.dumps(line))
    kd.shutdown()


if __name__ == "__main__":
    main()
