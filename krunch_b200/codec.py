"""GPU compress / decompress engine over one device-resident RWKV-4 model.

Compress (replaces krunch/inference.py:_compress_chunk_cpp 293-361 and the
batched variant 576-667): B chunks go through the packed forward together in
windows of Tw tokens (state carried across windows, so the window size never
changes a bit); each window's logits become (lo, hi) intervals of the actual
next tokens (kb_cdf_rows, LOHI mode) and every stream's range coder consumes
its rows lane-per-stream (kb_coder_encode_lohi).  The full [rows, V+1] CDF is
never built.

Decompress (replaces _decompress_chunks_batched_cpp, inference.py:363-443):
B chunks step in lock-step, one token per step: the T = 1 forward (same
kernels as compress, hence bit-identical logits) followed by the fused
softmax -> CDF -> search -> range-decoder step (kb_decode_logits_step).
Decoded tokens never leave the GPU until the end; after the first eager step
the whole step is captured once in a CUDA graph and replayed.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

from . import _native as N
from .model import RWKVModel

BOS_TOKEN = 0      # krunch/inference.py:98
TAIL_PAD = 64      # zero bytes after each bitstream (inference.py:403-419)


def max_code_bytes(n_tokens: int, cdf_bits: int) -> int:
    """Upper bound of one stream's encoded size: a symbol of width >= 1 in a
    total of 2^bits narrows the range by at most 2^bits plus rounding, i.e. < bits+2 bits,
    plus the final flush."""
    return (n_tokens * (cdf_bits + 2) + 64 + 7) // 8 + 16


_PER_BATCH_MEMORY_BYTES = 1.5 * 1024 * 1024   # krunch/cpp_path.py:528


def compute_decompress_batch(n_chunks: int = -1, device=None, default: int = 64) -> int:
    """Lock-step decompress batch B, the formula of krunch/cpp_path.py:531-580:
    env KRUNCH_DECOMPRESS_BATCH overrides (clamped to n_chunks); else
    SMs x 8 on sm >= 80 (SMs x 2 below), capped by 80 % of device memory at
    1.5 MiB per stream, and by n_chunks.  Without a CUDA device: ``default``.

    On B200 this gives 148 x 8 = 1184 streams.  A stream here holds 184 KB of
    fp32 state, a 100.6 KB numerator row, 12.6 KB of partials and ~70 KB of
    fused-step workspace (~370 KB), inside the reference's 1.5 MiB budget, so
    the reference's cap carries over unchanged."""
    env = os.environ.get("KRUNCH_DECOMPRESS_BATCH")
    if env:
        try:
            B = max(1, int(env))
            return min(n_chunks, B) if n_chunks > 0 else B
        except ValueError:
            pass
    try:
        if not torch.cuda.is_available():
            return default if n_chunks <= 0 else max(1, min(n_chunks, default))
        p = torch.cuda.get_device_properties(device if device is not None else 0)
        saturation = p.multi_processor_count * (8 if p.major >= 8 else 2)
        mem_cap = int(p.total_memory * 0.8 / _PER_BATCH_MEMORY_BYTES)
        upper = max(1, min(saturation, mem_cap))
    except Exception:
        upper = default
    if n_chunks > 0:
        return max(1, min(n_chunks, upper))
    return max(1, upper)


class Codec:
    def __init__(self, model: RWKVModel, cdf_bits: int = 24,
                 logits_budget_bytes: int = 8 << 30, use_graphs: bool | None = None):
        if not 2 <= cdf_bits <= 30 or (1 << cdf_bits) <= model.spec.n_vocab:
            raise ValueError(f"cdf_bits={cdf_bits} must give a total above the vocabulary")
        self.model = model
        self.bits = cdf_bits
        self.dev = model.device
        self.budget = logits_budget_bytes
        if use_graphs is None:
            use_graphs = N.env_flag("KRUNCH_CUDA_GRAPH", "1")
        self.use_graphs = use_graphs

    # ------------------------------------------------------------- compress
    def window_for(self, B: int, T: int) -> int:
        Vp = self.model.spec.vocab_pad
        env = os.environ.get("KRUNCH_FORWARD_BATCH")
        if env:
            return max(1, min(T, int(env)))
        tw = max(1, self.budget // (B * Vp * 2))
        if tw >= 64:
            tw -= tw % 64
        return max(1, min(T, tw))

    def compress_tokens(self, seqs: list[np.ndarray], max_batch: int | None = None) -> list[bytes]:
        """Encode each token sequence; returns one bitstream per sequence."""
        if not seqs:
            return []
        mb = max_batch or int(os.environ.get("KRUNCH_COMPRESS_BATCH", "1024"))
        out: list[bytes] = []
        for i in range(0, len(seqs), mb):
            out.extend(self._compress_group(seqs[i:i + mb]))
        return out

    def compress_batches(self, batches):
        """Pipelined compress of an iterable of batches (each a list of token
        sequences): yields each batch's bitstreams in order.  Batch i+1 is
        planned, uploaded and enqueued while batch i still runs on the GPU;
        batch i's results come back through pinned memory behind its own
        launches, so waiting for them does not wait for batch i+1."""
        prev = None
        for seqs in batches:
            plan = CompressPlan(self, [len(s) for s in seqs])
            plan.upload(seqs)
            plan.run()
            plan.fetch_async()
            if prev is not None:
                yield prev.fetch()
            prev = plan
        if prev is not None:
            yield prev.fetch()

    def _compress_group(self, seqs) -> list[bytes]:
        plan = CompressPlan(self, [len(s) for s in seqs])
        plan.upload(seqs)
        plan.run()
        return plan.fetch()

    def encode_window(self, logits, stats, sym_w, lohi, B, tw, n_valid, out_d, offs_d,
                      ac) -> None:
        """(lo, hi) of every row's symbol, then lane-per-stream encode."""
        m, s = self.model, N.stream_ptr(self.dev)
        N.call("kb_cdf_rows", logits.data_ptr(), m.spec.vocab_pad, B * tw, m.spec.n_vocab,
               self.bits, N.KB_CDF_LOHI, stats.data_ptr(), m.stats_stride, sym_w.data_ptr(),
               lohi.data_ptr(), s)
        N.call("kb_coder_encode_lohi", lohi.data_ptr(), B, tw, n_valid.data_ptr(), self.bits,
               out_d.data_ptr(), out_d.numel(), offs_d.data_ptr(), ac.data_ptr(), s)

    # ----------------------------------------------------------- decompress
    def decompress_tokens(self, streams: list[bytes], n_tokens: list[int],
                          max_batch: int | None = None) -> list[np.ndarray]:
        if not streams:
            return []
        mb = max_batch or compute_decompress_batch(len(streams), self.dev)
        out: list[np.ndarray] = []
        for i in range(0, len(streams), mb):
            out.extend(self._decompress_group(streams[i:i + mb], n_tokens[i:i + mb]))
        return out

    def _decompress_group(self, streams, ns) -> list[np.ndarray]:
        plan = DecompressPlan(self, [len(b) for b in streams], ns)
        plan.upload(streams)
        plan.run()
        return plan.fetch()


class CompressPlan:
    """Device buffers and launches for compressing B streams of given lengths.

    upload() copies the token ids (through pinned host memory), run() enqueues
    the whole compress on the current stream with every input resident in
    HBM, fetch() copies the bitstreams back.  h2d_bytes / d2h_bytes count the
    bytes those copies move."""

    def __init__(self, codec: "Codec", lens):
        self.codec = codec
        m, dev, bits = codec.model, codec.dev, codec.bits
        self.B = B = len(lens)
        self.lens = np.asarray(lens, dtype=np.int64)
        self.Tmax = Tmax = int(max(1, self.lens.max()))
        self.caps = np.array([(max_code_bytes(int(n), bits) + 15) // 16 * 16 for n in self.lens],
                             np.int64)
        self.offs = np.concatenate([[0], np.cumsum(self.caps)[:-1]]).astype(np.int64)
        self.total = int(self.caps.sum())
        self.inp_d = torch.empty((B, Tmax), dtype=torch.int32, device=dev)
        self.tgt_d = torch.empty((B, Tmax), dtype=torch.int32, device=dev)
        self.lens_d = torch.from_numpy(self.lens.astype(np.int32)).to(dev)
        self.offs_d = torch.from_numpy(self.offs).to(dev)
        self.out_d = torch.zeros(self.total, dtype=torch.uint8, device=dev)
        self.ac = torch.empty(B * 4, dtype=torch.int32, device=dev)
        self.Tw = codec.window_for(B, Tmax)
        self.state = m.new_state(B)
        self.ws = m.new_workspace(B, self.Tw)
        self.logits = m.new_logits(B, self.Tw)
        self.stats = m.new_stats(B, self.Tw)
        self.lohi = torch.empty((B, self.Tw, 2), dtype=torch.int32, device=dev)
        self.windows = (Tmax + self.Tw - 1) // self.Tw
        self._pin = torch.empty((2, B, Tmax), dtype=torch.int32).pin_memory()
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def upload(self, seqs) -> None:
        V = self.codec.model.spec.n_vocab
        host = self._pin.numpy()
        host[:] = 0
        for b, s in enumerate(seqs):
            s = np.asarray(s, dtype=np.int64)
            if s.size and (s.min() < 0 or s.max() >= V):
                raise ValueError(f"token id outside [0, {V})")
            n = s.size
            host[1, b, :n] = s
            host[0, b, 1:n] = s[:-1]
        self.inp_d.copy_(self._pin[0], non_blocking=True)
        self.tgt_d.copy_(self._pin[1], non_blocking=True)
        self.h2d_bytes = 2 * self._pin[0].numel() * 4

    def set_device_tokens(self, targets: torch.Tensor) -> None:
        """Targets already in HBM ([B, Tmax] int32): inputs = [BOS] + targets[:-1]."""
        self.tgt_d.copy_(targets)
        self.inp_d[:, 0] = BOS_TOKEN
        self.inp_d[:, 1:] = targets[:, :-1]

    def run(self) -> None:
        c, m = self.codec, self.codec.model
        s = N.stream_ptr(c.dev)
        self.out_d.zero_()
        N.call("kb_coder_encode_init", self.ac.data_ptr(), self.B, s)
        N.call("kb_state_init", m.handle, self.state.data_ptr(), self.B, s)
        for off in range(0, self.Tmax, self.Tw):
            tw = min(self.Tw, self.Tmax - off)
            if tw == self.Tmax:
                tok_w, sym_w = self.inp_d, self.tgt_d
            else:
                tok_w = self.inp_d[:, off:off + tw].contiguous()
                sym_w = self.tgt_d[:, off:off + tw].contiguous()
            m.forward_window(tok_w, self.state, self.ws, self.logits, self.stats)
            c.encode_window(self.logits, self.stats, sym_w, self.lohi, self.B, tw,
                            (self.lens_d - off).clamp(0, tw).int(), self.out_d, self.offs_d,
                            self.ac)
        N.call("kb_coder_encode_finalize", self.out_d.data_ptr(), self.total,
               self.offs_d.data_ptr(), self.ac.data_ptr(), self.B, s)

    def launches_per_run(self) -> int:
        """Kernels of this library that run() launches."""
        m = self.codec.model
        L = m.spec.n_layer
        # LN1, grouped k/v/r, WKV, att out, LN2, ffn receptance, ffn key,
        # ffn value (+ 2 row quantisations for w8a8)
        per_layer = 10 if m.spec.wdtype == "i8" else 8
        per_window = 1 + per_layer * L + 2 + 2   # embed, layers, ln_out+head, cdf+encode
        return 2 + self.windows * per_window + 1

    def fetch_async(self) -> None:
        """Enqueue the copies of the coder states and bitstreams into pinned
        host memory behind run() on the current stream, and record an event;
        fetch() then waits for that event only, not for later work."""
        self._ac_h = torch.empty(self.ac.shape, dtype=self.ac.dtype).pin_memory()
        self._out_h = torch.empty(self.out_d.shape, dtype=self.out_d.dtype).pin_memory()
        self._ac_h.copy_(self.ac, non_blocking=True)
        self._out_h.copy_(self.out_d, non_blocking=True)
        self._done = torch.cuda.Event()
        self._done.record(torch.cuda.current_stream(self.codec.dev))

    def fetch(self) -> list[bytes]:
        if getattr(self, "_done", None) is not None:
            self._done.synchronize()
            ac_h = self._ac_h.numpy().view(np.uint32).reshape(self.B, 4)
            out_h = self._out_h.numpy()
            self._done = None
        else:
            ac_h = self.ac.view(self.B, 4).cpu().numpy().view(np.uint32)
            out_h = self.out_d.cpu().numpy()
        self.d2h_bytes = self.ac.numel() * 4 + self.out_d.numel()
        res = []
        for b in range(self.B):
            nbytes = (int(ac_h[b, 3]) + 7) // 8
            if nbytes > self.caps[b]:
                raise RuntimeError(f"stream {b}: encoded size {nbytes} exceeds its buffer")
            res.append(out_h[self.offs[b]:self.offs[b] + nbytes].tobytes())
        return res


class DecompressPlan:
    """Device buffers and the lock-step decode loop for B streams.

    upload() stages the concatenated bitstreams (64 zero bytes after each),
    run() decodes every stream to its token count on the GPU (CUDA graph
    after the first step), fetch() returns the tokens."""

    def __init__(self, codec: "Codec", stream_bytes, n_tokens):
        self.codec = codec
        m, dev = codec.model, codec.dev
        self.B = B = len(n_tokens)
        self.ns = [int(n) for n in n_tokens]
        self.Tmax = max(self.ns) if self.ns else 0
        self.offs, pos = [], 0
        for n in stream_bytes:
            self.offs.append(pos)
            pos += int(n) + TAIL_PAD
        self.nbytes = max(pos, 1)
        self.in_d = torch.zeros(self.nbytes, dtype=torch.uint8, device=dev)
        self.offs_d = torch.tensor(self.offs, dtype=torch.int64, device=dev)
        self.ac = torch.empty(B * 4, dtype=torch.int32, device=dev)
        self.counters = torch.tensor([[0, n] for n in self.ns], dtype=torch.int32, device=dev)
        self.history = torch.zeros((B, max(self.Tmax, 1)), dtype=torch.int32, device=dev)
        self.cur = torch.zeros((B, 1), dtype=torch.int32, device=dev)
        self.state = m.new_state(B)
        self.fused = m.has_fused_step and N.env_flag("KRUNCH_FUSED_STEP", "1")
        self.ws = m.new_step_workspace(B) if self.fused else m.new_workspace(B, 1)
        self.logits = m.new_logits(B, 1)
        self.stats = m.new_stats(B, 1)
        self.graph = None
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def upload(self, streams) -> None:
        cat = torch.zeros(self.nbytes, dtype=torch.uint8).pin_memory()
        h = cat.numpy()
        for o, bs in zip(self.offs, streams):
            h[o:o + len(bs)] = np.frombuffer(bs, np.uint8)
        self.in_d.copy_(cat, non_blocking=True)
        self.h2d_bytes = self.nbytes

    def _step(self) -> None:
        c, m = self.codec, self.codec.model
        if self.fused:
            m.step_forward(self.cur.view(-1), self.state, self.ws, self.logits, self.stats)
        else:
            m.forward_window(self.cur, self.state, self.ws, self.logits, self.stats)
        N.call("kb_decode_logits_step", self.logits.data_ptr(), m.spec.vocab_pad, self.B,
               m.spec.n_vocab, c.bits, self.stats.data_ptr(), m.stats_stride, self.in_d.data_ptr(),
               self.nbytes, self.offs_d.data_ptr(),
               self.ac.data_ptr(), self.counters.data_ptr(), self.cur.data_ptr(),
               self.history.data_ptr(), self.history.shape[1], N.stream_ptr(c.dev))

    def run(self) -> None:
        c, m = self.codec, self.codec.model
        s = N.stream_ptr(c.dev)
        N.call("kb_coder_decode_init", self.in_d.data_ptr(), self.nbytes, self.offs_d.data_ptr(),
               self.ac.data_ptr(), self.B, s)
        N.call("kb_state_init", m.handle, self.state.data_ptr(), self.B, s)
        self.counters[:, 0] = 0
        self.cur.zero_()
        for t in range(self.Tmax):
            if self.graph is not None:
                self.graph.replay()
            elif t >= 1 and c.use_graphs and self.Tmax > 2:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._step()
                self.graph = g
                g.replay()
            else:
                self._step()

    def launches_per_run(self) -> int:
        m = self.codec.model
        if self.fused:
            return 2 + self.Tmax * 3  # fused layers, head, decode
        per_layer = 10 if m.spec.wdtype == "i8" else 8
        return 2 + self.Tmax * (1 + per_layer * m.spec.n_layer + 2 + 1)

    def fetch(self) -> list[np.ndarray]:
        hist = self.history.cpu().numpy()
        self.d2h_bytes = self.history.numel() * 4
        return [hist[b, :n].copy() for b, n in enumerate(self.ns)]


def bits_per_byte(blob_len: int, raw_len: int) -> float:
    return 8.0 * blob_len / raw_len if raw_len else math.nan
