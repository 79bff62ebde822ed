"""Benchmark of the NKIPy -> B200 path on the benchmark configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl nkb|reference]

A step is one execution of the traced kernel body of the workload on its
full-size seeded synthetic inputs, resident in HBM.  Rank 0 prints one JSON
line.  Workloads (``--workload``):

  softmax  fp32 (4096, 4096) row softmax                    HBM GB/s
  rmsnorm  fp32 (16384, 4096) residual add + RMSNorm         HBM GB/s
  gemm     bf16 8192^3 matmul, fp32 accumulate               TFLOP/s
  bmm      bf16 32 x 2048^3 batched matmul                   TFLOP/s
  linattn  bf16 (8, 16, 4096, 128) chunked linear attention  HBM GB/s
  layer    Llama decoder layer, batch 4 x 2048, TP = N       tokens/s
  decode   Qwen3 attention decode step, KV cache resident    tokens/s
  topk     top-8 of (128, 151936) bf16 logits                HBM GB/s
  conv     conv2d bf16 3x3, (16, 128, 56, 56)                TFLOP/s
  ewchain  fp32 (16384, 4096) silu(gate) * up                HBM GB/s
  transpose fp32 (8192, 8192) materialised transpose         HBM GB/s

Timing: W untimed warm-up steps, then K steps each preceded by an L2 flush
(256 MiB written, then read back, outside the timed events: the lines it
leaves in L2 are clean, so no write-back of the flush falls inside the timed
step) and timed with CUDA events
on the plan's stream; barrier + synchronize on both sides; the max over
ranks is reported.  ``e2e`` repeats the K steps through the public API with
pinned host buffers: H2D of each step's inputs, execute, D2H of the result.
A step's inputs are all the kernel's inputs, except for the decoder layer,
whose weights, norm weights and rotary tables are model parameters uploaded
once and kept on the device (as the reference's decode loop keeps its layer
weights as device tensors, examples/models/qwen3/qwen3.py:280-336); there
only the activations ``x`` move per step.
``--impl reference`` times the CPU path of the same kernel (the NumPy
direct call restated in ``oracle/``) on a bounded sample, on rank 0 only.

Parity: after the timed regions, rank 0 reads the outputs back and compares a
bounded sample with the oracle (the checker, never the thing measured), at
every GPU count: for the decoder layer the first 256 tokens of sequence 0,
which by causality depend only on that sequence's first 256 input tokens.
The line's ``parity`` object (and each suite entry's) says whether it held.
"""

import argparse
import concurrent.futures
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import ml_dtypes  # noqa: E402

BF16 = np.dtype(ml_dtypes.bfloat16)
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def flush_l2(buf):
    """Evict L2: write a buffer larger than L2, then read it back so that the
    lines left behind are clean (no write-back of the flush inside the next
    timed step)."""
    import torch

    buf.zero_()
    buf.view(torch.int32).sum()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def compare(got, want, rtol, sample, exact=False):
    """Parity of a device result against the oracle on a bounded sample, with
    the tests' criteria: bit-exact for integer/index work; fp32 elementwise
    ``|d| <= rtol |want| + 1e-7 max(1, max|want|)``; bf16 paths normwise
    ``|d| <= rtol max|want|``."""
    if exact:
        got, want = np.asarray(got), np.asarray(want)
        if got.dtype == want.dtype:  # bit patterns (floats: the sign of zero and NaNs included)
            ok = got.shape == want.shape and bool(np.array_equal(np.ascontiguousarray(got).view(np.uint8),
                                                                 np.ascontiguousarray(want).view(np.uint8)))
        else:
            ok = got.shape == want.shape and bool(np.array_equal(got, want))
        return {"ok": ok, "max_rel_err": 0.0 if ok else None, "tol": "exact", "sample": sample}
    g, w = np.asarray(got).astype(np.float32), np.asarray(want).astype(np.float32)
    peak = max(1e-30, float(np.max(np.abs(w)))) if w.size else 1.0
    d = np.abs(g - w)
    err = float(np.max(d)) / peak if d.size else 0.0
    if rtol <= 1e-5:
        ok = bool(np.all(d <= rtol * np.abs(w) + 1e-7 * max(1.0, peak)))
    else:
        ok = bool(err <= rtol)
    ok = ok and bool(np.all(np.isfinite(g)))
    return {"ok": ok, "max_rel_err": err, "tol": rtol, "sample": sample}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
class Workload:
    name = ""
    metric = ""
    unit = ""
    bound = "hbm"
    dtype = "f32"
    scaling = "weak"
    dominant = ""
    # kernel inputs copied host -> device every e2e step (None: all of them);
    # the others are parameters uploaded once
    step_inputs = None
    # outputs read back every e2e step (None: all of them)
    step_outputs = None

    def kernel_and_args(self, rank, world):
        raise NotImplementedError

    def units_per_step(self, world):
        raise NotImplementedError

    def dominant_work(self):
        """Algorithmic bytes (hbm) or flops (tensor) of one dominant launch."""
        raise NotImplementedError

    def cpu_prepare(self):
        """Inputs of the bounded CPU sample, built once outside the timed steps."""
        return ()

    def cpu_inputs(self):
        if getattr(self, "_cpu_in", None) is None:
            self._cpu_in = self.cpu_prepare()
        return self._cpu_in

    def cpu_step(self, threads):
        """One bounded CPU sample on ``cpu_inputs()``: returns (units processed, description)."""
        raise NotImplementedError

    def config(self, world):
        return {}

    def parity(self, outs, args):
        """Compare the device outputs (output name -> ndarray) with the oracle on
        a bounded sample of the inputs ``args``; returns the ``compare`` record."""
        return None


class Softmax(Workload):
    name, metric, unit, bound, dtype, dominant = "softmax", "HBM GB/s (row softmax)", "GB/s", "hbm", "f32", "softmax_rows"
    ROWS, COLS = 4096, 4096

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        x = np.random.default_rng(100 + rank).standard_normal((self.ROWS, self.COLS), dtype=np.float32)
        return W.softmax_kernel, (x,), {}

    def units_per_step(self, world):
        return 2 * self.ROWS * self.COLS * 4 / 1e9

    def dominant_work(self):
        return 2 * self.ROWS * self.COLS * 4

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        (x,) = self.cpu_inputs()
        rows = x.shape[0]
        _parallel_rows(O.softmax, [x], threads)
        return 2 * rows * self.COLS * 4 / 1e9, f"{rows} of {self.ROWS} rows per step"

    def cpu_prepare(self):
        return (np.random.default_rng(7).standard_normal((1024, self.COLS), dtype=np.float32),)

    def config(self, world):
        return {"workload": "softmax fp32 (4096, 4096) last axis", "shape": [self.ROWS, self.COLS],
                "l2": "flushed between steps (256 MiB written, then read back)"}

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        x = args[0][:256]
        return compare(outs["output0"][:256], O.softmax(x), 1e-5, "rows 0..255")


class RmsNorm(Workload):
    name, metric, unit, bound, dtype, dominant = "rmsnorm", "HBM GB/s (residual add + RMSNorm)", "GB/s", "hbm", "f32", "rmsnorm_rows"
    ROWS, COLS = 16384, 4096

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        rng = np.random.default_rng(200 + rank)
        x = rng.standard_normal((self.ROWS, self.COLS), dtype=np.float32)
        r = rng.standard_normal((self.ROWS, self.COLS), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, self.COLS).astype(np.float32)
        return W.residual_rmsnorm_kernel, (x, r, w), {}

    def units_per_step(self, world):
        return (3 * self.ROWS * self.COLS * 4 + self.COLS * 4) / 1e9

    def dominant_work(self):
        return 3 * self.ROWS * self.COLS * 4 + self.COLS * 4

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        x, r, w = self.cpu_inputs()
        rows = x.shape[0]
        _parallel_rows(lambda a, b: O.residual_rmsnorm(a, b, w, 1e-6), [x, r], threads)
        return (3 * rows * self.COLS * 4 + self.COLS * 4) / 1e9, f"{rows} of {self.ROWS} rows per step"

    def cpu_prepare(self):
        rng = np.random.default_rng(8)
        x = rng.standard_normal((2048, self.COLS), dtype=np.float32)
        r = rng.standard_normal((2048, self.COLS), dtype=np.float32)
        return x, r, rng.uniform(0.5, 1.5, self.COLS).astype(np.float32)

    def config(self, world):
        return {"workload": "residual add + RMSNorm fp32 (16384, 4096), eps 1e-6", "shape": [self.ROWS, self.COLS],
                "l2": "inputs (805 MB) exceed L2; also flushed between steps"}

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        x, r, w = args
        return compare(outs["output0"][:256], O.residual_rmsnorm(x[:256], r[:256], w, 1e-6), 1e-5, "rows 0..255")


class Gemm(Workload):
    name, metric, unit, bound, dtype, dominant = "gemm", "bf16 TFLOP/s (dense matmul)", "TFLOP/s", "tensor", "bf16", "gemm_bf16"
    N = 8192

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        rng = np.random.default_rng(300 + rank)
        a = (rng.standard_normal((self.N, self.N), dtype=np.float32) * 0.02).astype(BF16)
        b = (rng.standard_normal((self.N, self.N), dtype=np.float32) * 0.02).astype(BF16)
        return W.matmul_kernel, (a, b), {}

    def units_per_step(self, world):
        return 2 * self.N**3 / 1e12

    def dominant_work(self):
        return 2 * self.N**3

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        a, b = self.cpu_inputs()
        m = a.shape[0]
        O.matmul(a, b)
        return 2 * m * self.N * self.N / 1e12, f"{m} of {self.N} rows of A per step (fp32 BLAS, {threads} threads)"

    def cpu_prepare(self):
        rng = np.random.default_rng(9)
        a = (rng.standard_normal((1024, self.N), dtype=np.float32) * 0.02).astype(BF16)
        return a, (rng.standard_normal((self.N, self.N), dtype=np.float32) * 0.02).astype(BF16)

    def config(self, world):
        return {"workload": "matmul bf16 (8192,8192)@(8192,8192), fp32 acc, bf16 out", "M": self.N, "N": self.N,
                "K": self.N, "l2": "operands+result 384 MB exceed L2; also flushed between steps"}

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        a, b = args
        return compare(outs["output0"][:128], O.matmul(a[:128], b), 2e-2, "rows 0..127")


class Bmm(Gemm):
    name, metric, dominant = "bmm", "bf16 TFLOP/s (batched matmul)", "gemm_bf16"
    B, S = 32, 2048

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        rng = np.random.default_rng(400 + rank)
        a = (rng.standard_normal((self.B, self.S, self.S), dtype=np.float32) * 0.02).astype(BF16)
        b = (rng.standard_normal((self.B, self.S, self.S), dtype=np.float32) * 0.02).astype(BF16)
        return W.bmm_kernel, (a, b), {}

    def units_per_step(self, world):
        return 2 * self.B * self.S**3 / 1e12

    def dominant_work(self):
        return 2 * self.B * self.S**3

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        a, b = self.cpu_inputs()
        O.matmul(a, b)
        return 2 * 2 * self.S**3 / 1e12, f"2 of {self.B} batches per step"

    def cpu_prepare(self):
        rng = np.random.default_rng(10)
        a = (rng.standard_normal((2, self.S, self.S), dtype=np.float32) * 0.02).astype(BF16)
        return a, (rng.standard_normal((2, self.S, self.S), dtype=np.float32) * 0.02).astype(BF16)

    def config(self, world):
        return {"workload": "batched matmul bf16 bmk,bkn->bmn b=32 m=n=k=2048", "batch": self.B, "M": self.S,
                "l2": "operands 805 MB exceed L2; also flushed between steps"}

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        a, b = args
        return compare(outs["output0"][31], O.matmul(a[31], b[31]), 2e-2, "batch 31")


class LinAttn(Workload):
    name, metric, unit, bound, dtype, dominant = "linattn", "HBM GB/s (chunked causal linear attention)", "GB/s", "hbm", "bf16", "linattn"
    SHAPE = (8, 16, 4096, 128)

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        q, k, v = W.make_inputs("linattn", seed=600 + rank)
        return W.chunked_linear_attention_kernel, (q, k, v), {}

    def units_per_step(self, world):
        return 4 * int(np.prod(self.SHAPE)) * 2 / 1e9

    def dominant_work(self):
        return 4 * int(np.prod(self.SHAPE)) * 2

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        q, k, v = self.cpu_inputs()
        O.linear_attention_recurrent(q, k, v)
        return 4 * q.size * 2 / 1e9, "1 x 2 of 8 x 16 (batch, head) pairs per step"

    def cpu_prepare(self):
        from nkipy_b200 import workloads as W

        q, k, v = W.make_inputs("linattn", seed=7, scale=1 / 8)
        return tuple(np.ascontiguousarray(t[:, :2]) for t in (q, k, v))

    def config(self, world):
        return {"workload": "chunked causal linear attention bf16 (8,16,4096,128), elu+1, chunk 64, fp32 state",
                "shape": list(self.SHAPE), "l2": "inputs 403 MB exceed L2; also flushed between steps"}

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        q, k, v = args
        sl = (slice(7, 8), slice(15, 16))
        return compare(outs["output0"][sl], O.linear_attention_recurrent(q[sl], k[sl], v[sl]), 2e-2,
                       "(batch, head) (7, 15)")


class Layer(Workload):
    name, metric, unit, bound, dtype, dominant = "layer", "TP decoder layer tokens/s", "tokens/s", "tensor", "bf16", "gemm_bf16"
    scaling = "strong"
    step_inputs = ("x",)

    def __init__(self):
        from nkipy_b200 import workloads as W

        self.shape = W.LayerShape()

    PREFIX = 256  # tokens of sequence 0 in the CPU sample and the parity check

    def _full(self):
        from nkipy_b200 import workloads as W

        if getattr(self, "_weights", None) is None:
            s = self.shape
            self._weights = W.layer_weights(s, seed=0)
            self._x = np.random.default_rng(500).standard_normal((s.batch, s.seq, s.hidden),
                                                                 dtype=np.float32).astype(BF16)
        return self._weights, self._x

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        s = self.shape
        full, x = self._full()
        shard = W.shard_layer_weights(full, s, rank, world)
        args, kwargs = W.layer_args(x, shard, s, world)
        return W.llama_decoder_layer_kernel, args, kwargs

    def units_per_step(self, world):
        return self.shape.batch * self.shape.seq

    def layer_flops(self):
        s = self.shape
        t = s.batch * s.seq
        hd = s.head_dim
        f = 2 * t * s.hidden * (s.n_heads + 2 * s.n_kv_heads) * hd + 2 * t * s.n_heads * hd * s.hidden
        f += 2 * t * s.hidden * 2 * s.ffn + 2 * t * s.ffn * s.hidden
        f += 0.5 * 4 * s.batch * s.n_heads * s.seq * s.seq * hd
        return f

    def dominant_work(self):
        return None  # computed from the per-launch table

    def _oracle_prefix(self, seq=0):
        """The oracle's layer on the first PREFIX tokens of sequence ``seq`` of the bench input."""
        from oracle import numpy_ref as O

        full, x = self._full()
        s = self.shape
        return O.llama_layer(x[seq : seq + 1, : self.PREFIX], full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps,
                             s.theta)

    def cpu_prepare(self):
        return self._full()

    def cpu_step(self, threads):
        self.cpu_inputs()
        self._oracle_prefix()
        return self.PREFIX, f"1 x {self.PREFIX} tokens of the layer per step (sequence 0, tokens 0..{self.PREFIX - 1})"

    def parity(self, outs, args):
        # output tokens 0..PREFIX-1 of a sequence depend only on its input tokens 0..PREFIX-1 (causal
        # attention); the first and the last sequence (under TP with the e2e row split, the last one's
        # input reached rank 0 through the all-gather)
        y = outs["output0"]
        last = self.shape.batch - 1
        a = compare(y[:1, : self.PREFIX], self._oracle_prefix(0), 2e-2, "")
        b = compare(y[last : last + 1, : self.PREFIX], self._oracle_prefix(last), 2e-2, "")
        return {"ok": a["ok"] and b["ok"], "max_rel_err": max(a["max_rel_err"], b["max_rel_err"]), "tol": 2e-2,
                "sample": f"sequences 0 and {last}, tokens 0..{self.PREFIX - 1} (causal prefixes) of the full-shape run"}

    def sampling_parity(self, rank, world):
        """Vocabulary-parallel greedy sampling (examples/models/qwen3/kernels/sampling.py:113-147) at this
        world size: top-1 per rank, all-gather of the ranks' maxima and ids, top-1 over the ranks.  Every
        rank runs it (collectives inside); rank 0 checks the ids."""
        from nkipy_b200 import workloads as W
        from nkipy_b200.runtime import DeviceKernel, DeviceTensor

        B, S, H, V = 4, 8, 4096, 32000
        rng = np.random.default_rng(17)
        h = rng.standard_normal((B, S, H), dtype=np.float32).astype(BF16)
        nw = rng.uniform(0.5, 1.5, H).astype(BF16)
        lm = (rng.standard_normal((H, V), dtype=np.float32) * 0.05).astype(BF16)
        shard = np.ascontiguousarray(lm[:, rank * (V // world) : (rank + 1) * (V // world)])
        k = DeviceKernel.compile_and_load(W.greedy_sampling_kernel, h, nw, shard, name="bench_sampling",
                                          is_spmd=False, cc_enabled=True, rank_id=rank, world_size=world,
                                          max_batch_size=B, tp_world=world)
        names = [t["name"] for t in k.model_ref.io["inputs"]]
        outs = k(inputs={n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, (h, nw, shard))})
        ids = next(iter(outs.values())).numpy().reshape(-1).astype(np.int64)
        if rank != 0:
            return None
        logits = W.qk_rmsnorm(h, nw, 1e-6)[:, -1, :].astype(np.float32) @ lm.astype(np.float32)
        best = logits.max(axis=1)
        picked = logits[np.arange(B), np.clip(ids, 0, V - 1)]
        # the chosen token holds the largest logit up to the bf16 rounding of the device's logits
        ok = bool(np.all((ids >= 0) & (ids < V)) and np.all(picked >= best - (2.0**-7 * np.abs(best) + 1e-6)))
        return {"ok": ok, "ids": ids.tolist(), "sample": f"greedy sampling, vocabulary {V} split over {world} ranks"}

    def config(self, world):
        s = self.shape
        return {"workload": "Llama decoder layer bf16, hidden 4096, 32q/8kv x 128, SwiGLU 14336, RoPE 5e5, causal",
                "global_batch": s.batch, "seq_len": s.seq, "parallelism": f"tp{world}",
                "l2": "weights + activations exceed L2"}


class Decode(Workload):
    """One decode step of the Qwen3 attention block with its KV cache resident
    and updated in place (examples/models/qwen3/kernels/attention.py:25-156,
    qwen3.py:280-336): 8 sequences, cache length 2048, hidden 4096, 32 query /
    8 KV heads of 128.  Bound by HBM: the step reads the projection weights
    and both caches once; the roofline is taken over the whole step."""

    name, metric, unit, bound, dtype, dominant = "decode", "decode tokens/s (KV-cache attention step)", "tokens/s", "hbm", "bf16", "*step*"
    B, L, H, NQ, NKV, HD = 8, 2048, 4096, 32, 8, 128
    step_inputs = ("x", "start_pos")  # weights and caches stay resident between steps
    step_outputs = ("output0",)  # the caches are updated in place on the device

    def _args(self, B, seed):
        from nkipy_b200 import workloads as W

        rng = np.random.default_rng(seed)
        x = rng.standard_normal((B, 1, self.H), dtype=np.float32).astype(BF16)
        wqkv = (rng.standard_normal((self.H, (self.NQ + 2 * self.NKV) * self.HD), dtype=np.float32) * 0.02).astype(BF16)
        wo = (rng.standard_normal((self.NQ * self.HD, self.H), dtype=np.float32) * 0.02).astype(BF16)
        qn = rng.uniform(0.5, 1.5, self.HD).astype(BF16)
        kn = rng.uniform(0.5, 1.5, self.HD).astype(BF16)
        ck = rng.standard_normal((B, self.L, self.NKV, self.HD), dtype=np.float32).astype(BF16)
        cv = rng.standard_normal((B, self.L, self.NKV, self.HD), dtype=np.float32).astype(BF16)
        pos = np.array([self.L - 1], np.int32)
        kw = dict(n_heads=self.NQ, head_dim=self.HD, n_kv_heads=self.NKV)
        return W.cached_attention_kernel, (x, wqkv, qn, kn, ck, cv, pos, wo), kw

    def kernel_and_args(self, rank, world):
        return self._args(self.B, 700 + rank)

    def units_per_step(self, world):
        return self.B

    def dominant_work(self):
        # projection weights + both caches read once, the new token's cache rows written
        w = self.H * (self.NQ + 2 * self.NKV) * self.HD * 2 + self.NQ * self.HD * self.H * 2
        return w + 2 * self.B * self.L * self.NKV * self.HD * 2

    def cpu_prepare(self):
        return self._args(1, 11)

    def cpu_step(self, threads):
        fn, args, kw = self.cpu_inputs()
        # the caches are mutated in place by the direct call: work on copies
        args = tuple(a.copy() if isinstance(a, np.ndarray) else a for a in args)
        fn(*args, **kw)
        return 1, f"1 of {self.B} sequences per step (NumPy direct call)"

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        fn, _, kw = self._args(self.B, 700)
        # sequence 0 alone, on copies of its original inputs (the device caches
        # were updated in place at the same position by every timed step)
        x, wqkv, qn, kn, ck, cv, pos, wo = self._args(self.B, 700)[1]
        with O.fp32_accumulated_bf16_sums():  # long bf16 softmax sums, accumulated in fp32 as on the device
            want = fn(x[:1].copy(), wqkv, qn, kn, ck[:1].copy(), cv[:1].copy(), pos, wo, **kw)
        return compare(outs["output0"][:1], want, 2e-2, "sequence 0 of 8")

    def config(self, world):
        return {"workload": "Qwen3 attention decode step bf16, KV cache 2048 resident and updated in place, "
                            "hidden 4096, 32q/8kv x 128", "batch": self.B, "cache_len": self.L,
                "l2": "weights + caches 149 MB exceed L2; also flushed between steps"}


class TopK(Workload):
    """Last-axis top-8 of 128 rows of a Qwen3 vocabulary (151936) in bf16: the
    sampling step (core/ops/nn.py:65-152).  Bound by HBM on the logits read."""

    name, metric, unit, bound, dtype, dominant = "topk", "HBM GB/s (top-8 over a vocabulary)", "GB/s", "hbm", "bf16", "topk_rows"
    ROWS, COLS, K = 128, 151936, 8

    def kernel_and_args(self, rank, world):
        from nkipy_b200.core.ops import nn

        x = np.random.default_rng(800 + rank).standard_normal((self.ROWS, self.COLS), dtype=np.float32).astype(BF16)

        def topk_kernel(logits):
            return nn.topk(logits, self.K, axis=-1)

        return topk_kernel, (x,), {}

    def units_per_step(self, world):
        return self.ROWS * self.COLS * 2 / 1e9

    def dominant_work(self):
        return self.ROWS * self.COLS * 2

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        (x,) = self.cpu_inputs()
        O.topk(x, self.K)
        return x.shape[0] * self.COLS * 2 / 1e9, f"{x.shape[0]} of {self.ROWS} rows per step"

    def cpu_prepare(self):
        return (np.random.default_rng(12).standard_normal((16, self.COLS), dtype=np.float32).astype(BF16),)

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        vals, idx = O.topk(args[0][:16], self.K)
        a = compare(outs["output1"][:16], idx, 0, "rows 0..15", exact=True)
        b = compare(outs["output0"][:16], vals, 0, "rows 0..15", exact=True)
        return {**a, "ok": a["ok"] and b["ok"]}

    def config(self, world):
        return {"workload": "top-8 bf16 (128, 151936) last axis", "shape": [self.ROWS, self.COLS], "k": self.K,
                "l2": "flushed between steps"}


class Conv(Workload):
    """conv2d bf16, batch 16, 128 -> 128 channels, 3x3, padding 1 on 56x56
    (core/ops/conv.py): pad, kernel windows written dense, one GEMM."""

    name, metric, unit, bound, dtype, dominant = "conv", "bf16 TFLOP/s (conv2d 3x3)", "TFLOP/s", "tensor", "bf16", "gemm_bf16"
    B, C, OC, HW = 16, 128, 128, 56

    def kernel_and_args(self, rank, world):
        from nkipy_b200.core import ops as OPS

        rng = np.random.default_rng(900 + rank)
        x = rng.standard_normal((self.B, self.C, self.HW, self.HW), dtype=np.float32).astype(BF16)
        w = (rng.standard_normal((self.OC, self.C, 3, 3), dtype=np.float32) * 0.05).astype(BF16)

        def conv_kernel(x, w):
            return OPS.conv2d(x, w, stride=1, padding=1)

        return conv_kernel, (x, w), {}

    def units_per_step(self, world):
        return 2 * self.B * self.OC * self.C * 9 * self.HW * self.HW / 1e12

    def dominant_work(self):
        return 2 * self.B * self.OC * self.C * 9 * self.HW * self.HW

    def cpu_step(self, threads):
        from oracle import numpy_ref as O

        x, w = self.cpu_inputs()
        O.conv_nd(x, w, padding=1)
        return 2 * self.OC * self.C * 9 * self.HW * self.HW / 1e12, f"1 of {self.B} images per step"

    def cpu_prepare(self):
        rng = np.random.default_rng(13)
        x = rng.standard_normal((1, self.C, self.HW, self.HW), dtype=np.float32).astype(BF16)
        return x, (rng.standard_normal((self.OC, self.C, 3, 3), dtype=np.float32) * 0.05).astype(BF16)

    def parity(self, outs, args):
        from oracle import numpy_ref as O

        x, w = args
        return compare(outs["output0"][15:16], O.conv_nd(x[15:16], w, padding=1), 2e-2, "image 15 of 16")

    def config(self, world):
        return {"workload": "conv2d bf16 x(16,128,56,56) w(128,128,3,3) padding 1",
                "l2": "flushed between steps"}


class EwChain(Workload):
    """silu(gate) * up over fp32 (16384, 4096): one fused elementwise chain
    (the SwiGLU activation, examples/models/qwen3_embedding/kernels/ffn.py)."""

    name, metric, unit, bound, dtype, dominant = "ewchain", "HBM GB/s (fused elementwise chain)", "GB/s", "hbm", "f32", "ew"
    ROWS, COLS = 16384, 4096

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        rng = np.random.default_rng(1000 + rank)
        g = rng.standard_normal((self.ROWS, self.COLS), dtype=np.float32)
        u = rng.standard_normal((self.ROWS, self.COLS), dtype=np.float32)
        return W.silu_mul_kernel, (g, u), {}

    def units_per_step(self, world):
        return 3 * self.ROWS * self.COLS * 4 / 1e9

    def dominant_work(self):
        return 3 * self.ROWS * self.COLS * 4

    def cpu_prepare(self):
        rng = np.random.default_rng(14)
        return tuple(rng.standard_normal((2048, self.COLS), dtype=np.float32) for _ in range(2))

    def cpu_step(self, threads):
        from nkipy_b200 import workloads as W

        g, u = self.cpu_inputs()
        _parallel_rows(W.silu_mul_kernel, [g, u], threads)
        return 3 * g.size * 4 / 1e9, f"{g.shape[0]} of {self.ROWS} rows per step (NumPy direct call)"

    def parity(self, outs, args):
        from nkipy_b200 import workloads as W

        g, u = args
        return compare(outs["output0"][:256], W.silu_mul_kernel(g[:256], u[:256]), 1e-5, "rows 0..255")

    def config(self, world):
        return {"workload": "silu(gate) * up fp32 (16384, 4096)", "shape": [self.ROWS, self.COLS],
                "l2": "inputs 537 MB exceed L2; also flushed between steps"}


class Transpose(Workload):
    """np.transpose of fp32 (8192, 8192), materialised (core/ops/transform.py:55-79)."""

    name, metric, unit, bound, dtype, dominant = "transpose", "HBM GB/s (materialised transpose)", "GB/s", "hbm", "f32", "transpose_tiles"
    N = 8192

    def kernel_and_args(self, rank, world):
        from nkipy_b200 import workloads as W

        x = np.random.default_rng(1100 + rank).standard_normal((self.N, self.N), dtype=np.float32)
        return W.transpose_kernel, (x,), {}

    def units_per_step(self, world):
        return 2 * self.N * self.N * 4 / 1e9

    def dominant_work(self):
        return 2 * self.N * self.N * 4

    def cpu_prepare(self):
        return (np.random.default_rng(15).standard_normal((2048, self.N), dtype=np.float32),)

    def cpu_step(self, threads):
        (x,) = self.cpu_inputs()
        # column blocks of the transposed result, one per thread
        out = np.empty((x.shape[1], x.shape[0]), np.float32)
        bounds = np.linspace(0, x.shape[1], threads + 1).astype(int)

        def part(i):
            out[bounds[i]:bounds[i + 1]] = x[:, bounds[i]:bounds[i + 1]].T

        with concurrent.futures.ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(part, range(threads)))
        return 2 * x.size * 4 / 1e9, f"{x.shape[0]} of {self.N} rows per step"

    def parity(self, outs, args):
        return compare(outs["output0"], np.ascontiguousarray(args[0].T), 0, "whole output", exact=True)

    def config(self, world):
        return {"workload": "transpose fp32 (8192, 8192) materialised", "shape": [self.N, self.N],
                "l2": "input 268 MB exceeds L2; also flushed between steps"}


WORKLOADS = {w.name: w for w in (Softmax, RmsNorm, Gemm, Bmm, LinAttn, Layer, Decode, TopK, Conv, EwChain, Transpose)}
DEFAULT_WORKLOAD = "layer"
SUITE = ("softmax", "rmsnorm", "gemm", "bmm", "linattn", "decode", "topk", "conv", "ewchain", "transpose")


def _parallel_rows(fn, arrays, threads):
    n = arrays[0].shape[0]
    chunks = max(1, min(threads, n))
    bounds = np.linspace(0, n, chunks + 1).astype(int)
    with concurrent.futures.ThreadPoolExecutor(max_workers=chunks) as ex:
        list(ex.map(lambda i: fn(*[a[bounds[i] : bounds[i + 1]] for a in arrays]), range(chunks)))


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        # samples go to a private temporary file (NKB_CLOCKS_CSV keeps them at a chosen path)
        self.keep = os.environ.get("NKB_CLOCKS_CSV")
        self.path = self.keep or os.path.join(tempfile.mkdtemp(prefix="nkb_clocks_"), f"gpu{gpu_index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 9:
                    continue
                try:
                    sm.append(float(p[1]))
                    mx = max(mx, float(p[2]))
                except ValueError:
                    continue
                for n, v in zip(names, p[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        if not self.keep:
            shutil.rmtree(os.path.dirname(self.path), ignore_errors=True)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------
def cpu_measure(wl, steps, warmup, threads):
    for _ in range(warmup):
        wl.cpu_step(threads)
    units, t, desc = 0.0, 0.0, ""
    for _ in range(steps):
        t0 = time.perf_counter()
        u, desc = wl.cpu_step(threads)
        t += time.perf_counter() - t0
        units += u
    return units / t, desc, t / steps


def run_reference(args, wl, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    value, desc, step_s = cpu_measure(wl, args.steps, max(0, min(args.warmup, 1)), threads)
    line = {
        "impl": "reference",
        "metric": wl.metric,
        "value": value,
        "unit": wl.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_s * 1e3,
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic (seeded numpy), bounded sample",
        "config": wl.config(world),
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def profile_traffic(wl):
    """dram bytes per launch of the dominant kernel (the whole step for the decode
    step) from the committed ncu summary."""
    stem = "attn_decode" if wl.dominant == "*step*" else wl.dominant
    p = os.path.join(ROOT, "profiles", f"{stem}_{wl.name}.md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


def _tensor_numpy(spike, t, spec):
    """A device buffer read back as the plan io spec's array."""
    import ml_dtypes as md

    dt = np.dtype(md.bfloat16) if spec["dtype"] == "bfloat16" else np.dtype(spec["dtype"])
    raw = np.frombuffer(spike.tensor_read(t), dtype=np.uint8)
    n = int(np.prod(spec["shape"], dtype=np.int64)) * dt.itemsize
    return raw[:n].view(dt).reshape(spec["shape"])


def _outputs_numpy(kernel, outs):
    """Every plan output read back to the host (name -> ndarray)."""
    return {s["name"]: outs[s["name"]].numpy() for s in kernel.model_ref.io["outputs"]}


def _roofline(wl, plan_steps, step_ms, ms_per_step, peaks, peak_kind):
    """Roofline record of the dominant kernel: algorithmic work per launch over its
    mean CUDA-event launch time inside the timed graph replays
    (``nkb_time_execute_steps``), against the measured peak.  The timed region
    is short (tens of ms of steps, each after an L2 flush), so GEMMs are set
    against the burst bf16 figure."""
    dom = [i for i, st in enumerate(plan_steps) if st["kernel"] == wl.dominant]
    if wl.dominant == "*step*":
        # no single dominant launch (the decode step): the whole step's algorithmic
        # bytes over the device-timed step
        peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        achieved = wl.dominant_work() / (ms_per_step / 1e3) / 1e9
        return {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": None, "peak_source": f"{peak_kind} (hbm_gbs)", "kernel": "whole step",
                "launch_ms": ms_per_step, "work_per_launch": wl.dominant_work()}
    if not dom:
        return None
    dur = sum(step_ms[i] for i in dom) / len(dom)
    if wl.bound == "hbm":
        work = wl.dominant_work()
        achieved, key, unit = work / (dur / 1e3) / 1e9, "hbm_gbs", "GB/s"
    else:
        work = sum(plan_steps[i]["flops"] for i in dom) / len(dom)
        achieved, key, unit = work / (dur / 1e3) / 1e12, "bf16_tflops", "TFLOP/s"
    peak = float(peaks.get(key, PEAKS_FALLBACK[key]))
    return {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": None, "peak_source": f"{peak_kind} ({key})", "kernel": wl.dominant, "launch_ms": dur,
            "work_per_launch": work}


def run_nkb(args, wl, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    os.environ["NKB_DEVICE"] = str(local_rank)
    torch.cuda.set_device(local_rank)
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor
    from nkipy_b200.spike import get_spike_singleton

    spike = get_spike_singleton()
    fn, np_args, kwargs = wl.kernel_and_args(rank, world)
    cc = world > 1 and wl.name == "layer"
    kernel = DeviceKernel.compile_and_load(
        fn, *np_args, name=f"bench_{wl.name}", cc_enabled=cc, rank_id=rank if cc else None,
        world_size=world if cc else None, is_spmd=False, **kwargs
    )
    in_names = [s["name"] for s in kernel.model_ref.io["inputs"]]
    arrays = [a for a in np_args if isinstance(a, np.ndarray)]
    ins = {n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(in_names, arrays)}
    # a mutated input (``<name>.must_alias_input``, the KV caches) is bound in place as its output
    outs = {t.name: ins.get(f"{t.name}.must_alias_input", t) for t in kernel.allocate_output_tensors()}
    in_refs = {k: v.tensor_ref for k, v in ins.items()}
    out_refs = {k: v.tensor_ref for k, v in outs.items()}
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=f"cuda:{local_rank}")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local_rank}")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # clocks are sampled from the start of warm-up to the end of the e2e region
    sampler = ClockSampler(local_rank)
    sampler.start()
    # Each timed step replays the plan's CUDA graph (its time is the step's), then,
    # after another L2 flush, the same plan with an event between every two
    # launches: the dominant kernel's launch times come from inside the timed
    # region, while the event nodes (a few microseconds per step) stay out of the
    # step's time.  The decode step's roofline is the whole step: no second replay.
    per_launch = wl.dominant != "*step*"
    for _ in range(args.warmup):
        spike.execute(kernel.model_ref, in_refs, out_refs, use_graph=True)
        if per_launch:
            spike.time_execute_steps(kernel.model_ref, in_refs, out_refs)
    barrier()
    total_ms = 0.0
    step_acc = [0.0] * kernel.model_ref.num_launches
    for _ in range(args.steps):
        flush_l2(flush)
        # every rank's flush is done before any rank starts the step, so the
        # collectives inside it do not time another rank's flush
        barrier()
        total_ms += spike.time_execute(kernel.model_ref, in_refs, out_refs, warmup=0, iters=1, use_graph=True)[0]
        if per_launch:
            flush_l2(flush)
            barrier()
            _, per = spike.time_execute_steps(kernel.model_ref, in_refs, out_refs)
            step_acc = [a + b for a, b in zip(step_acc, per)]
    barrier()
    total_ms = max_over_ranks(total_ms)
    ms_per_step = total_ms / args.steps

    # per-launch times (the roofline of the dominant kernel): inside the timed
    # steps, else launch by launch after them
    if per_launch:
        step_ms = [a / args.steps for a in step_acc]
    else:
        step_ms = spike.time_steps(kernel.model_ref, in_refs, out_refs, iters=max(3, min(args.steps, 10)))
    plan_steps = _plan_steps(kernel.plan_path)

    # End to end through the public API, pinned host memory.  Per step the job
    # uploads every step input once and reads every step output once.  For the
    # tensor-parallel layer (N > 1) the token rows are split across the ranks:
    # rank r uploads its 1/N of x's rows, an in-place all-gather over NVLink
    # gives every rank the whole x, and after the execute rank r reads back its
    # 1/N of y's rows; whole-job bytes crossing the host boundary are the same
    # as at N = 1.
    step_names = [n for n in in_names if wl.step_inputs is None or n in wl.step_inputs]
    step_arrays = [a for n, a in zip(in_names, arrays) if n in step_names]
    out_specs = [s for s in kernel.model_ref.io["outputs"] if wl.step_outputs is None or s["name"] in wl.step_outputs]
    split = cc and kernel.model_ref.comm is not None and all(
        a.nbytes % world == 0 for a in step_arrays) and all(
        outs[s["name"]].tensor_ref.size % world == 0 for s in out_specs)
    parts = world if split else 1
    part = rank if split else 0
    pinned_in = []
    for a in step_arrays:
        n = a.nbytes // parts
        p = torch.empty(n, dtype=torch.uint8, pin_memory=True).numpy()
        p[:] = np.ascontiguousarray(a).reshape(-1).view(np.uint8)[part * n : (part + 1) * n]
        pinned_in.append(p)
    pinned_out = [torch.empty(outs[s["name"]].tensor_ref.size // parts, dtype=torch.uint8, pin_memory=True).numpy()
                  for s in out_specs]
    # the public pipelined API: each step's upload and read-back overlap the
    # neighbouring steps' compute (two device buffer sets, three streams)
    resident = {n: ins[n] for n in in_names if n not in step_names}
    host_in = dict(zip(step_names, pinned_in))
    host_out = {sp["name"]: p for sp, p in zip(out_specs, pinned_out)}
    bind = {name: t for name, t in outs.items() if f"{name}.must_alias_input" in ins}
    kernel.run_steps(resident, host_in, host_out, 2, split=split, bind=bind)  # buffers, graphs
    barrier()
    t0 = time.perf_counter()
    e2e_outs = kernel.run_steps(resident, host_in, host_out, args.steps, split=split, bind=bind)
    # kernels one execute launches: the kernel nodes of the plan's CUDA graph (a
    # step may launch none, e.g. a copy onto itself, one or two)
    kg = kernel.model_ref.graph_kernels
    kernels_per_step = kg if kg >= 0 else kernel.model_ref.num_launches
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks = sampler.stop()

    # parity of the full-shape run against the oracle (rank 0 checks, the others wait)
    parity = None
    if rank == 0 and not args.no_parity:
        try:
            # the last end-to-end step's outputs (under the TP row split its input was
            # completed by the all-gather)
            got = {sp["name"]: _tensor_numpy(spike, e2e_outs[sp["name"]], sp) for sp in kernel.model_ref.io["outputs"]}
            parity = wl.parity(got, arrays)
        except Exception as e:  # report, never hide, a failing check
            parity = {"ok": False, "error": f"{type(e).__name__}: {e}"}
    barrier()
    if cc and not args.no_parity:
        # the vocabulary-parallel sampling step with its all-gathers, on every rank
        samp = wl.sampling_parity(rank, world)
        if rank == 0:
            parity = dict(parity or {}, sampling=samp)
            parity["ok"] = bool(parity.get("ok")) and bool(samp and samp.get("ok"))
        barrier()

    units = wl.units_per_step(world)
    if wl.scaling == "weak":
        value = world * units * args.steps / (total_ms / 1e3)
        e2e_value = world * units * args.steps / e2e_s
    else:
        value = units * args.steps / (total_ms / 1e3)
        e2e_value = units * args.steps / e2e_s

    if rank != 0:
        return
    peaks, peak_kind = load_peaks()
    roof = _roofline(wl, plan_steps, step_ms, ms_per_step, peaks, peak_kind)
    if roof is not None and world == 1:
        roof["traffic"] = profile_traffic(wl)  # the committed ncu summaries are single-GPU captures

    cpu = None
    if world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        cv, desc, _ = cpu_measure(wl, 2, 1, threads)
        cpu = {"value": cv, "unit": wl.unit, "cores": threads, "kind": "port", "sample": desc}

    in_bytes = int(sum(a.nbytes for a in step_arrays))
    resident = [n for n in in_names if n not in step_names]
    out_bytes = int(sum(outs[s["name"]].tensor_ref.size for s in out_specs))
    e2e = {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes}
    if split:
        e2e["split"] = (f"whole-job bytes; rank r uploads 1/{world} of the step inputs' rows, all-gathers them "
                        f"in place over NVLink, and reads back 1/{world} of the output rows")
    if resident:
        e2e["resident_bytes"] = int(sum(a.nbytes for n, a in zip(in_names, arrays) if n in resident))
    line = {
        "metric": wl.metric,
        "value": value,
        "unit": wl.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic (seeded numpy; random-init weights for the layer)",
        "config": wl.config(world),
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": kernels_per_step * args.steps,
        "clocks": clocks,
        "launches_per_step": kernels_per_step,
        "plan_steps": kernel.model_ref.num_launches,
        "per_launch_ms": {f"{i}:{st['kernel']}": round(ms, 4) for i, (st, ms) in enumerate(zip(plan_steps, step_ms))}
        if len(step_ms) <= 24 else None,
    }
    if world == 1 and not args.no_suite:
        suite = {}
        for name in SUITE:
            if name == wl.name:
                continue
            try:
                suite[name] = measure_quick(WORKLOADS[name](), 5, 3, local_rank, not args.no_cpu, not args.no_parity)
            except Exception as e:  # report, never hide, a failing configuration
                suite[name] = {"error": f"{type(e).__name__}: {e}"}
        line["suite"] = suite
    # last, so that it stays in view at the end of a long line
    line["parity"] = parity
    print(json.dumps(line), flush=True)


def measure_quick(wl, steps, warmup, local_rank, with_cpu, with_parity):
    """Single-GPU measurement of one workload for the suite object (same method,
    fewer steps); a compact record: value, roofline fraction, CPU baseline, parity."""
    import torch

    from nkipy_b200.runtime import DeviceKernel, DeviceTensor
    from nkipy_b200.spike import get_spike_singleton

    spike = get_spike_singleton()
    fn, np_args, kwargs = wl.kernel_and_args(0, 1)
    kernel = DeviceKernel.compile_and_load(fn, *np_args, name=f"suite_{wl.name}", is_spmd=False, **kwargs)
    names = [t["name"] for t in kernel.model_ref.io["inputs"]]
    arrays = [a for a in np_args if isinstance(a, np.ndarray)]
    dins = {n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, arrays)}
    ins = {n: t.tensor_ref for n, t in dins.items()}
    # a mutated input (``<name>.must_alias_input``) is bound in place as its output
    douts = {t.name: dins.get(f"{t.name}.must_alias_input", t) for t in kernel.allocate_output_tensors()}
    outs = {n: t.tensor_ref for n, t in douts.items()}
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=f"cuda:{local_rank}")
    per_launch = wl.dominant != "*step*"  # as in run_nkb
    for _ in range(warmup):
        spike.execute(kernel.model_ref, ins, outs, use_graph=True)
        if per_launch:
            spike.time_execute_steps(kernel.model_ref, ins, outs)
    total = 0.0
    step_acc = [0.0] * kernel.model_ref.num_launches
    for _ in range(steps):
        flush_l2(flush)
        torch.cuda.synchronize()
        total += spike.time_execute(kernel.model_ref, ins, outs, warmup=0, iters=1, use_graph=True)[0]
        if per_launch:
            flush_l2(flush)
            torch.cuda.synchronize()
            _, per = spike.time_execute_steps(kernel.model_ref, ins, outs)
            step_acc = [a + b for a, b in zip(step_acc, per)]
    ms = total / steps
    if per_launch:
        step_ms = [a / steps for a in step_acc]
    else:
        step_ms = spike.time_steps(kernel.model_ref, ins, outs, iters=3)
    peaks, peak_kind = load_peaks()
    roof = _roofline(wl, _plan_steps(kernel.plan_path), step_ms, ms, peaks, peak_kind)
    out = {
        "value": round(wl.units_per_step(1) / (ms / 1e3), 4),
        "unit": wl.unit,
        "ms": round(ms, 4),
        "launches": kernel.model_ref.graph_kernels if kernel.model_ref.graph_kernels >= 0 else kernel.model_ref.num_launches,
        "frac": round(roof["frac"], 3) if roof else None,
    }
    if with_cpu:
        cv, _, _ = cpu_measure(wl, 1, 0, os.cpu_count() or 1)
        out["cpu"] = float(f"{cv:.4g}")
    if with_parity:
        try:
            par = wl.parity(_outputs_numpy(kernel, douts), arrays)
            out["parity"] = bool(par["ok"])
            if par.get("max_rel_err") is not None and par["tol"] != "exact":
                out["err"] = float(f"{par['max_rel_err']:.3g}")
        except Exception as e:  # report, never hide, a failing check
            out["parity"] = False
            out["err"] = f"{type(e).__name__}: {e}"[:120]
    del kernel, ins, outs, dins, douts
    return out


def _plan_steps(path):
    """Kernel name and flop count of every launch of a plan file."""
    out = []
    with open(path) as f:
        for line in f:
            if not line.startswith("step "):
                continue
            p = line.split()
            kern = p[1]
            nb = int(p[2])
            k = 3 + 2 * nb
            ni = int(p[k])
            ints = [int(v) for v in p[k + 1 : k + 1 + ni]]
            flops = 0
            if kern == "gemm_bf16":
                M, N, K, batch = ints[0], ints[1], ints[2], ints[6]
                if len(ints) == 15 and ints[13] == 1:  # SwiGLU epilogue: gate and up halves
                    N *= 2
                flops = 2 * M * N * K * batch
            elif kern == "gemm_simt":
                M, N, K, batch = ints[3], ints[4], ints[5], ints[6]
                flops = 2 * M * N * K * batch
            out.append({"kernel": kern, "flops": flops})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="nkb", choices=["nkb", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-suite", action="store_true", help="at N=1, skip measuring the other configurations")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity check against the oracle")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[args.workload]()
    if args.impl == "reference":
        return run_reference(args, wl, rank, world)
    # keep stdout to the one JSON line (NCCL prints a version banner at INFO/VERSION)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local_rank}"))
    try:
        run_nkb(args, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
