#!/usr/bin/env python
"""Benchmark: ms/layer of the FFTSparse prefill hot path at 128K tokens.

One step = one attention layer of BASELINE config 3: block mean pooling of q
and k, FFT-correlation block-mask selection and block-sparse causal attention
(the whole of myattn_prefill, attn_src/fft_attn/my_attn_v7.py:454-792) for
L = 131072 tokens, 32 query heads over 8 KV heads, head_dim 128, bf16, block
128, keep ratio 0.05, on seeded synthetic inputs (fftsparse_b200/synthetic.py).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1 calls the drop-in ``myattn_prefill`` with repeat_kv-expanded k/v, the
exact call of the reference's benchmark
(eval/efficiency/benchmark_attention_multilayer.py:146-157, :308).  N > 1
(launched by torchrun, one rank per GPU, NCCL) shards the 8 KV groups over the
ranks; the attention kernel's epilogue stores each output tile into every
peer's head-major buffer over NVLink, so the all-gather runs alongside the math
(fftsparse_b200/dist.py, PeerGather); total work is fixed, so the
scaling is strong.  ``--impl reference`` times the CPU
restatement of the reference path (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "ms/layer (FFT mask select + block-sparse attn) at 128k"
UNIT = "ms/layer"
SEQ_LEN = 131072
HQ, HKV, HEAD_DIM, BLOCK = 32, 8, 128, 128


def mask_kwargs(keep_ratio: float) -> dict:
    """Keep ratio r -> the reference's arguments (topk mode; efficiency-script ratios,
    eval/efficiency/1_run_eval_multilayer.sh:46-63, :72)."""
    return dict(block_size=BLOCK, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
                enable_correlation_mask=True, correlation_selection_mode="topk",
                correlation_topk_ratio=keep_ratio, corr_threshold=1.0, enable_column_mask=True,
                column_topk_ratio=0.2, enable_last_block_mask=True, diag_sample_ratio=0.15,
                min_diag_samples=5, max_diag_samples=64, qk_topk_ratio=keep_ratio,
                stripe_threshold=0.3)


def threshold_kwargs(threshold: float) -> dict:
    """Threshold-mode arguments of the reference's published efficiency run
    (eval/efficiency/1_run_eval_multilayer.sh:29-31, :46-60, :72;
    benchmark_attention_multilayer.py:301-303: correlation_topk_ratio 0.2 in
    threshold mode)."""
    return dict(block_size=BLOCK, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
                enable_correlation_mask=True, correlation_selection_mode="threshold",
                correlation_topk_ratio=0.2, corr_threshold=threshold, enable_column_mask=True,
                column_topk_ratio=0.2, enable_last_block_mask=True, diag_sample_ratio=0.15,
                min_diag_samples=5, max_diag_samples=64, qk_topk_ratio=0.3, stripe_threshold=0.3)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--keep-ratio", type=float, default=0.05)
    ap.add_argument("--seq-len", type=int, default=SEQ_LEN)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-ttft", action="store_true")
    ap.add_argument("--no-caller-kernels", action="store_true", help="skip the rope_pool / decode bandwidth fields")
    ap.add_argument("--ttft-layers", type=int, default=0, help="0: the config's own layer count")
    ap.add_argument("--ttft-config", type=int, choices=[4, 5], default=4,
                    help="BASELINE config of the TTFT decoder (4: Llama-3.1-8B shape, 1 x seq-len tokens; "
                         "5: Qwen2.5-7B shape, 2 x 65536 tokens, block 64)")
    ap.add_argument("--ttft-seq-len", type=int, default=0, help="config 5 sequence length (0: 65536)")
    ap.add_argument("--ttft-qkv", choices=["fused", "rope_pool"], default="fused",
                    help="QKV path of the TTFT decoder: qkv_rope_pool (projection GEMM with RoPE and pooling in "
                         "its epilogue) or a cuBLAS projection followed by rope_pool")
    ap.add_argument("--caller-kernels-only", action="store_true",
                    help="time only the caller-side kernels (qkv_rope_pool, rope_pool, decode) at --seq-len on one "
                         "GPU and print their field (the small case the profiles capture)")
    ap.add_argument("--clock-log", default="",
                    help="directory for the raw nvidia-smi clock samples (default: a temporary directory)")
    return ap.parse_args()


# ----------------------------------------------------------------- helpers
def load_peaks():
    """(HBM GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, kind) from MEASURED_PEAKS.json,
    else the pool's earlier measurement."""
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    except (OSError, ValueError, KeyError, TypeError):  # absent or malformed: the pool's earlier figures
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling around the timed region.

    The sampler is started (and its first sample awaited) before the warm-up and
    stopped after the last measurement; `mark_begin`/`mark_end` bracket the timed
    loop.  The summary uses the samples taken inside that window when there are
    any; a timed loop shorter than the sampling period (the 8-GPU layer takes a
    few ms) falls back to every sample taken under load during the bench and says
    so in `window`."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, log_dir: str = ""):
        import tempfile
        self.index = index
        self.proc = None
        self.path = os.path.join(log_dir or tempfile.mkdtemp(prefix="ffts_clocks_"), f"clocks_gpu{index}.csv")
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
            deadline = time.time() + 10.0  # nvidia-smi takes a moment to start
            while time.time() < deadline and os.path.getsize(self.path) == 0 and self.proc.poll() is None:
                time.sleep(0.02)
        except OSError:  # no nvidia-smi: the summary says so
            self.proc = None
        return self

    def mark_begin(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        from datetime import datetime
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]),
                             float(parts[4]) if parts[4] not in ("[N/A]", "") else 0.0, parts[6:10]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        window = "timed region"
        use = [r for r in rows if self.t0 is not None and self.t1 is not None and self.t0 <= r[0] <= self.t1]
        if not use:
            window = "whole bench under load (timed region shorter than the sampling period)"
            use = [r for r in rows if r[3] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i, v in enumerate(r[4]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(use), "window": window,
                "power_w": round(statistics.median(r[3] for r in use), 1)}


def causal_pairs(bits: torch.Tensor, L: int, bs: int) -> int:
    """Exact number of kept (query, key) pairs with key <= query."""
    B, H, N, W = bits.shape
    shifts = torch.arange(32, device=bits.device, dtype=torch.int64)
    dense = ((bits.to(torch.int64)[..., None] >> shifts) & 1).reshape(B, H, N, W * 32)[..., :N].to(torch.int64)
    sizes = torch.full((N,), bs, dtype=torch.int64, device=bits.device)
    sizes[-1] = L - (N - 1) * bs
    full = (dense * sizes[None, None, :, None] * sizes[None, None, None, :]).sum()
    diag = torch.diagonal(dense, dim1=2, dim2=3)  # [B, H, N]
    tri = sizes * (sizes + 1) // 2
    # replace the diagonal's rows*cols by the causal triangle
    corr = (diag * (tri - sizes * sizes)[None, None, :]).sum()
    return int(full + corr)


def own_kernel_launches(fn) -> int:
    """Launches of this library's kernels (names in the ffts:: namespace) during one
    call of ``fn``, from the CUDA activity trace (torch.profiler / CUPTI)."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return int(sum(ev.count for ev in prof.key_averages()
                   if ev.device_type is not None and not str(ev.device_type).endswith("CPU") and "ffts::" in ev.key))


def kernel_times_us(fn, reps: int = 3) -> dict:
    """Average device time per call of each kernel ``fn`` launches, in µs, from the
    CUDA activity trace of ``reps`` calls (torch.profiler / CUPTI); keys are the
    kernels' short names."""
    from torch.profiler import ProfilerActivity, profile
    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    out = {}
    for ev in prof.key_averages():
        if ev.device_type is None or str(ev.device_type).endswith("CPU"):
            continue
        name = ev.key.split("(")[0].split("<")[0].split("::")[-1]
        us = getattr(ev, "device_time_total", None)
        if us is None:
            us = getattr(ev, "cuda_time_total", 0.0)
        if us:
            out[name] = out.get(name, 0.0) + us / reps
    return {k: round(v, 2) for k, v in out.items()}


def caller_side_kernels(dev, L: int, hbm_peak: float, bf16_peak: float, reps: int = 5) -> dict:
    """The caller-side kernels at BASELINE config 4's shape (Llama-3.1-8B: hidden
    4096, 32 q / 8 KV heads of 128, L tokens):
    - qkv_rope_pool, the QKV projection GEMM with RoPE, layout and pooling in its
      epilogue: 2 x L x 4096 x 6144 FLOP against the measured bf16 peak, beside
      the unfused path it replaces (cuBLAS bf16 matmul, then rope_pool);
    - rope_pool on one layer's QKV projection, against HBM: it reads the
      projection (L x 6144 bf16) and cos / sin, writes q, k, v head-major and the
      pooled q / k blocks;
    - one decode step over an L-token cache of 8 KV heads, against HBM: it reads
      the K and V caches once (2 x L x 8 x 128 x 2 bytes)."""
    import fftsparse_b200 as F
    g = torch.Generator(device=dev).manual_seed(0)
    H, HKV_, D = HQ, HKV, HEAD_DIM
    qkv = torch.randn(L, (H + 2 * HKV_) * D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float64) / D))
    fr = torch.arange(L, device=dev, dtype=torch.float64)[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    del fr, emb

    def rp():
        return F.rope_pool(qkv[:, :H * D], qkv[:, H * D:(H + HKV_) * D], qkv[:, (H + HKV_) * D:], H, HKV_, cos, sin,
                           BLOCK)

    def timed(fn, n=reps):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    t_rp = timed(rp)
    N = (L + BLOCK - 1) // BLOCK
    rp_bytes = 2 * L * (H + 2 * HKV_) * D * 2 + 2 * L * D * 2 + N * (H + HKV_) * D * 2
    del qkv
    hid = 4096
    x = (torch.randn(L, hid, generator=g, device=dev, dtype=torch.float32)).to(torch.bfloat16)
    w = (torch.randn((H + 2 * HKV_) * D, hid, generator=g, device=dev, dtype=torch.float32) * hid ** -0.5).to(
        torch.bfloat16)
    t_fused = timed(lambda: F.qkv_rope_pool(x, w, None, H, HKV_, cos, sin, BLOCK))

    def unfused():
        qkv_ = torch.matmul(x, w.T)
        return F.rope_pool(qkv_[:, :H * D], qkv_[:, H * D:(H + HKV_) * D], qkv_[:, (H + HKV_) * D:], H, HKV_, cos,
                           sin, BLOCK)

    t_unfused = timed(unfused)
    t_gemm = timed(lambda: torch.matmul(x, w.T))
    F.check_status(dev)
    qkv_flops = 2.0 * L * hid * (H + 2 * HKV_) * D
    del x, w
    torch.cuda.empty_cache()
    kc = torch.randn(1, HKV_, L, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn(1, HKV_, L, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    qd = torch.randn(1, H, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    t_dec = timed(lambda: F.decode_attention(qd, kc, vc), max(reps, 20))  # a 0.1 ms kernel: more calls
    dec_bytes = 2 * L * HKV_ * D * 2
    del kc, vc
    torch.cuda.empty_cache()
    return {"qkv_rope_pool": {"ms": round(t_fused, 4), "flops": qkv_flops,
                              "tflops": round(qkv_flops / (t_fused * 1e-3) / 1e12, 1),
                              "frac_bf16": round(qkv_flops / (t_fused * 1e-3) / 1e12 / bf16_peak, 4),
                              "unfused_ms": round(t_unfused, 4), "cublas_gemm_ms": round(t_gemm, 4),
                              "unfused": "torch.matmul (cuBLAS bf16) then rope_pool",
                              "shape": f"x [L={L}, {hid}] @ W^T [{hid}, {(H + 2 * HKV_) * D}], block {BLOCK}"},
            "rope_pool": {"ms": round(t_rp, 4), "bytes": rp_bytes, "gbs": round(rp_bytes / (t_rp * 1e-3) / 1e9, 1),
                          "frac_hbm": round(rp_bytes / (t_rp * 1e-3) / 1e9 / hbm_peak, 4),
                          "shape": f"L={L}, projection [L, {(H + 2 * HKV_) * D}] bf16, block {BLOCK}"},
            "decode": {"ms": round(t_dec, 4), "bytes": dec_bytes, "gbs": round(dec_bytes / (t_dec * 1e-3) / 1e9, 1),
                       "frac_hbm": round(dec_bytes / (t_dec * 1e-3) / 1e9 / hbm_peak, 4),
                       "shape": f"one token, {H} q / {HKV_} KV heads, Lk={L}"}}


# ----------------------------------------------------------- CPU baseline
def cpu_baseline_sample(q, k, v, keep_ratio, row_stride=16):
    """Oracle port on the host cores: full-size mask selection for all heads
    (C, OpenMP) plus fp32 block-sparse attention for head 0 on every
    ``row_stride``-th query block, scaled to the whole layer by the exact ratio
    of kept (query, key) pairs."""
    from oracle import oracle as O  # the checker, timed here as the CPU baseline
    from fftsparse_b200.params import derive_mask_params

    torch.set_num_threads(os.cpu_count() or 1)
    kw = mask_kwargs(keep_ratio)
    L = q.shape[2]
    params = derive_mask_params(L, **kw)
    t0 = time.perf_counter()
    ref = O.prefill_mask(q, k, params)
    t_mask = time.perf_counter() - t0
    N = params.n_blocks
    mask = O.unpack_bits(ref["bits"], N)
    rows = list(range(0, N, row_stride))
    t0 = time.perf_counter()
    O.sparse_attention(q, k, v, mask, BLOCK, heads=[0], rows=rows)
    t_attn = time.perf_counter() - t0
    counts = ref["row_count"].to(torch.float64)  # kept blocks per (b, h, row)
    scale = float(counts.sum()) / float(counts[0, 0, rows].sum())
    ms = 1e3 * (t_mask + t_attn * scale)
    return ms, {"mask_s": t_mask, "attn_sample_s": t_attn, "attn_scale": scale, "rows_sampled": len(rows),
                "threads": torch.get_num_threads(), "cpu_count": os.cpu_count()}


def run_reference(args):
    """--impl reference: the CPU path on the host cores (rank 0 only).

    Each step runs a bounded sample of the layer on the host cores and the
    line's value is the measured time of that sample per step: the full mask
    selection for all heads (the C oracle, OpenMP) plus fp32 block-sparse
    attention for head 0 on every 16th query block.  The time the whole layer
    would take on the CPU, scaled from the sample by kept (query, key) blocks,
    is reported beside it as ``extrapolated_ms_per_layer``."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from fftsparse_b200.synthetic import make_inputs
    q, k, v = make_inputs(args.seq_len, num_q_heads=HQ, num_kv_heads=HKV, dtype=torch.bfloat16)
    times, extrap, info = [], [], {}
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ms_layer, info = cpu_baseline_sample(q, k, v, args.keep_ratio)
        step_ms = (time.perf_counter() - t0) * 1e3
        if i >= args.warmup:
            times.append(step_ms)
            extrap.append(ms_layer)
    value = sum(times) / len(times)
    sample = (f"per step, measured: the full {args.seq_len}-token mask selection for all {HQ} heads (C oracle, "
              f"{info['threads']} OpenMP threads) plus fp32 block-sparse attention for head 0 on "
              f"{info['rows_sampled']} evenly spaced query blocks of {args.seq_len // BLOCK}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"cfg3: L={args.seq_len}, Hq={HQ}, Hkv={HKV} (expanded), D={HEAD_DIM}, "
                               f"block {BLOCK}, keep ratio {args.keep_ratio}; CPU sample of the layer (see "
                               f"cpu_baseline.sample)", "seq_len": args.seq_len,
                   "global_batch": 1, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": info.get("threads"),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "extrapolated_ms_per_layer": round(sum(extrap) / len(extrap), 1),
        "extrapolation": {"mask_s": round(info["mask_s"], 4), "attn_sample_s": round(info["attn_sample_s"], 4),
                          "attn_scale": round(info["attn_scale"], 2),
                          "how": "mask time + attention sample time x (kept blocks of all heads / kept blocks "
                                 "of the sampled query blocks of head 0)"},
        "detail": info,
    }
    emit(line)


# ------------------------------------------------------------- TTFT (cfg 4)
class DecoderShape:
    """Random-init decoder with the shapes of BASELINE configs 4 and 5, bf16.

    ``LLAMA31_8B`` (config 4): hidden 4096, 32 q / 8 kv heads of 128, SwiGLU
    14336, RMSNorm, RoPE base 500000, vocab 128256, 32 layers.  ``QWEN25_7B``
    (config 5): hidden 3584, 28 q / 4 kv heads of 128, SwiGLU 18944, RoPE base
    1e6, vocab 152064, 28 layers (shape only: no QKV bias).  Weights ~ N(0, 0.02)
    drawn with one seed (identical on every rank), norm weights 1.  The dense
    parts are torch/cuBLAS.  Per layer: RMSNorm; fftsparse_b200's qkv_rope_pool
    (the QKV projection GEMM with the caller's RoPE, the head-major layout and the
    pooling of q and k in its epilogue), or with ``qkv="rope_pool"`` a cuBLAS
    projection followed by rope_pool per sequence; its attention on un-expanded
    GQA k/v, given the pooled blocks.

    With world > 1 the layer is split two ways:
    - attention by (sequence, KV group) unit (unit_shard): each rank computes
      its units' QKV columns for its sequences and runs attention for its heads;
      the head-major output is all-gathered (in the attention epilogue when a
      PeerGather is given and the batch is one sequence, else NCCL);
    - o_proj and the MLP by token rows: each rank takes its contiguous slice of
      the B * L rows of the gathered output, applies o_proj, the residual,
      RMSNorm and the MLP to them, and one all-gather of the hidden states gives
      every rank all rows for the next layer's QKV projection.
    ``dims`` overrides (H, HKV, D, HIDDEN, INTER, VOCAB) for small test models."""

    LLAMA31_8B = dict(dims=(32, 8, 128, 4096, 14336, 128256), rope_base=500000.0, layers=32)
    QWEN25_7B = dict(dims=(28, 4, 128, 3584, 18944, 152064), rope_base=1e6, layers=28)

    def __init__(self, layers, device, world=1, rank=0, seed=0, gather=None, dims=None, batch=1,
                 rope_base=500000.0, qkv="fused"):
        from fftsparse_b200.dist import unit_shard
        self.H, self.HKV, self.D, self.HIDDEN, self.INTER, self.VOCAB = dims or self.LLAMA31_8B["dims"]
        self.B, self.rope_base = batch, rope_base
        if qkv not in ("fused", "rope_pool"):
            raise ValueError(f"qkv must be 'fused' or 'rope_pool', got {qkv!r}")
        self.qkv = qkv
        g = torch.Generator(device=device).manual_seed(seed)
        self.shard = unit_shard(batch, self.H, self.HKV, world, rank)
        self.world, self.rank = world, rank
        self.gather = gather  # dist.PeerGather of the (H, L) output, or None for NCCL
        D = self.D

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)

        sh = self.shard
        cols = torch.cat([torch.arange(sh.h_lo * D, sh.h_hi * D),
                          self.H * D + torch.arange(sh.kv_lo * D, sh.kv_hi * D),
                          (self.H + self.HKV) * D + torch.arange(sh.kv_lo * D, sh.kv_hi * D)]).to(device)
        self.embed = w(self.VOCAB, self.HIDDEN)
        self.layers = []
        for _ in range(layers):
            wqkv = w(self.HIDDEN, (self.H + 2 * self.HKV) * D).T  # Linear layout [out, in]
            self.layers.append(dict(
                wqkv=wqkv.contiguous() if world == 1 else wqkv[cols].contiguous(),
                wo=w(self.H * D, self.HIDDEN),
                wgu=w(self.HIDDEN, 2 * self.INTER),
                wd=w(self.INTER, self.HIDDEN)))
            del wqkv
        self.lm_head = w(self.HIDDEN, self.VOCAB)
        self.device = device
        self._rope = None

    @staticmethod
    def rmsnorm(x, eps=1e-5):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)

    def forward(self, ids, kw):
        """ids [B, L] (or [L] for one sequence) -> logits [B, VOCAB] of each sequence's
        last position."""
        import torch.distributed as dist

        import fftsparse_b200 as F
        from fftsparse_b200.dist import sharded_prefill
        ids = ids.view(self.B, -1)
        B, L = ids.shape
        D, H, INTER, HID = self.D, self.H, self.INTER, self.HIDDEN
        sh = self.shard
        Hl, Hkvl = sh.heads, sh.kv_hi - sh.kv_lo
        b_lo, b_hi = sh.b_lo, (B if sh.b_hi == -1 else sh.b_hi)  # this rank's sequences
        T = B * L
        if T % self.world:
            raise ValueError(f"{B} x {L} token rows do not split over {self.world} ranks")
        r0, r1 = self.rank * (T // self.world), (self.rank + 1) * (T // self.world)  # this rank's rows
        bs = kw.get("block_size", 128)
        if self._rope is None or self._rope[0].shape[0] != L:
            inv = 1.0 / (self.rope_base ** (torch.arange(0, D, 2, device=self.device, dtype=torch.float64) / D))
            fr = torch.arange(L, device=self.device, dtype=torch.float64)[:, None] * inv[None]
            emb = torch.cat([fr, fr], -1)
            self._rope = (emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16))
        cos, sin = self._rope

        def stack(ts):
            return ts[0] if len(ts) == 1 else torch.cat(ts, 0)

        h = self.embed[ids.reshape(-1)]  # [B * L, HID]
        for lw in self.layers:
            x = self.rmsnorm(h[b_lo * L:b_hi * L])
            if self.qkv == "fused":
                q, k, v, qb, kb = F.qkv_rope_pool(x.view(b_hi - b_lo, L, HID), lw["wqkv"], None, Hl, Hkvl, cos, sin,
                                                  bs)
                del x
            else:
                qkv = x @ lw["wqkv"].T
                del x
                parts = [F.rope_pool(qkv[i * L:(i + 1) * L, :Hl * D],
                                     qkv[i * L:(i + 1) * L, Hl * D:(Hl + Hkvl) * D],
                                     qkv[i * L:(i + 1) * L, (Hl + Hkvl) * D:], Hl, Hkvl, cos, sin, bs)
                         for i in range(b_hi - b_lo)]
                del qkv
                q, k, v, qb, kb = (stack([p[j] for p in parts]) for j in range(5))
                del parts
            if self.world == 1:
                attn = F.myattn_prefill(q, k, v, 0, pooled=(qb, kb), **kw).view(T, H * D)
            else:
                full = sharded_prefill(q, k, v, 0, inputs_are_local=True, global_batch=B, num_heads=H,
                                       num_kv_heads=self.HKV, gather=self.gather if B == 1 else None,
                                       pooled=(qb, kb), **kw)
                rows = []  # token rows [r0, r1) of the head-major output, token-major
                for b in range(B):
                    lo, hi = max(r0, b * L), min(r1, (b + 1) * L)
                    if lo < hi:
                        rows.append(full[b, :, lo - b * L:hi - b * L].transpose(0, 1).reshape(hi - lo, H * D))
                attn = stack(rows)
                del full, rows
            del q, k, v, qb, kb
            hr = h[r0:r1] + attn @ lw["wo"]
            del attn
            x = self.rmsnorm(hr)
            gu = x @ lw["wgu"]
            del x
            hr = hr + (torch.nn.functional.silu(gu[:, :INTER]) * gu[:, INTER:]) @ lw["wd"]
            del gu
            if self.world == 1:
                h = hr
            else:
                h = torch.empty_like(h)
                dist.all_gather_into_tensor(h, hr)
            del hr
        last = h.view(B, L, HID)[:, -1]
        return self.rmsnorm(last) @ self.lm_head  # logits of each sequence's last position


def run_ttft(args, dev, world, rank, stream, barrier, gather=None):
    """Prefill TTFT of BASELINE config 4 (default) or 5: token ids already on the
    device to the last positions' logits, device-timed with CUDA events, max over
    ranks."""
    import torch.distributed as dist
    if args.ttft_config == 5:
        shape, B, L, bs, name = DecoderShape.QWEN25_7B, 2, args.ttft_seq_len or 65536, 64, "cfg5: Qwen2.5-7B"
        gather = None  # two sequences: the NCCL gather
    else:
        shape, B, L, bs, name = DecoderShape.LLAMA31_8B, 1, args.seq_len, BLOCK, "cfg4: Llama-3.1-8B"
    layers = args.ttft_layers or shape["layers"]
    model = DecoderShape(layers, dev, world, rank, gather=gather, dims=shape["dims"], batch=B,
                         rope_base=shape["rope_base"], qkv=args.ttft_qkv)
    g = torch.Generator(device=dev).manual_seed(0)
    ids = torch.randint(0, model.VOCAB, (B, L), generator=g, device=dev)
    kw = dict(mask_kwargs(args.keep_ratio), block_size=bs)
    reps = 2
    with torch.no_grad():
        model.forward(ids, kw)
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            logits = model.forward(ids, kw)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    finite = bool(torch.isfinite(logits.float()).all())
    del model
    torch.cuda.empty_cache()
    return {"value": round(float(t.item()) / 1e3, 4), "unit": "s",
            "workload": f"{name}-shape decoder, {layers} layers, random N(0,0.02) weights "
                        f"(seed 0), bf16; prefill of {B} x {L} uniform random token ids (seed 0) to the last-token "
                        f"logits; FFTSparse attention (block {bs}, keep ratio {args.keep_ratio}) in every layer, "
                        f"GQA k/v un-expanded, "
                        + ("QKV projection GEMM with RoPE + layout + q/k pooling in its epilogue (qkv_rope_pool)"
                           if args.ttft_qkv == "fused" else
                           "cuBLAS QKV projection, then RoPE + layout + q/k pooling in one pass (rope_pool)")
                        + "; other dense parts torch/cuBLAS"
                        + ("" if world == 1 else f"; QKV columns and attention sharded by (sequence, KV group) over "
                                                 f"{world} ranks, o_proj/MLP sharded by token rows, hidden states "
                                                 f"all-gathered per layer"),
            "logits_finite": finite, "reps": reps}


# --------------------------------------------------------------- our arm
def run_ours(args):
    import torch.distributed as dist

    import fftsparse_b200 as F
    from fftsparse_b200.dist import PeerGather, kv_group_shard, local_views, sharded_prefill
    from fftsparse_b200.synthetic import make_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    F.load_library()
    kw = mask_kwargs(args.keep_ratio)
    L = args.seq_len

    # inputs: CPU draws (same values on every rank), RoPE and cast on the device
    q, k, v = make_inputs(L, num_q_heads=HQ, num_kv_heads=HKV, dtype=torch.bfloat16, device=str(dev))
    torch.cuda.synchronize(dev)

    # N > 1: the attention epilogue pushes the output rows to every peer over NVLink
    pg = PeerGather(HQ, L, HEAD_DIM, device=dev) if world > 1 else None

    def step():
        if world == 1:
            return F.myattn_prefill(q, k, v, 0, **kw)
        return sharded_prefill(q, k, v, 0, num_kv_heads=HKV, gather=pg, **kw)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # clocks are sampled from before the first warm-up step to the last measurement
    clocks = ClockSampler(local_rank, args.clock_log).__enter__()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    clocks.mark_begin()
    start.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to issue one step
    end.record(stream)
    torch.cuda.synchronize(dev)
    clocks.mark_end()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    # by construction: 2 pool + the range check + 3 selection kernels + attention, and at
    # N > 1 one flag store and one bounded wait; at N = 1 counted from the activity trace
    launches_per_step = 7 if world == 1 else 9
    if world == 1:
        try:  # an activity trace that saw nothing (no CUPTI, e.g. under ncu) keeps the count
            launches_per_step = own_kernel_launches(step) or launches_per_step
        except Exception:  # noqa: BLE001 - the trace is a report; keep the count by construction
            pass
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # ---- the same layer with un-expanded GQA k/v (8 KV heads): identical outputs,
    # the 4 q-heads of a group then share K/V tiles in L2
    k8 = k[:, ::HQ // HKV].contiguous()
    v8 = v[:, ::HQ // HKV].contiguous()
    for _ in range(2):
        F.myattn_prefill(q, k8, v8, 0, **kw) if world == 1 else sharded_prefill(q, k8, v8, 0, gather=pg, **kw)
    torch.cuda.synchronize(dev)
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(args.steps):
        F.myattn_prefill(q, k8, v8, 0, **kw) if world == 1 else sharded_prefill(q, k8, v8, 0, gather=pg, **kw)
    g1.record(stream)
    torch.cuda.synchronize(dev)
    tg = torch.tensor([g0.elapsed_time(g1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
    gqa_native_ms = float(tg.item())
    del k8, v8

    # ---- per-stage timing and the attention kernel's roofline (rank-local shard)
    shard = kv_group_shard(HQ, HKV, world, rank)
    ql, kl, vl = local_views(q, k, v, shard)
    mask = F.fft_block_mask(ql, kl, **kw)
    torch.cuda.synchronize(dev)
    barrier()  # no rank still pushes rows of the previous loop into this one's memory
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    reps = max(3, args.steps)
    ev[0].record(stream)
    for _ in range(reps):
        F.pool_blocks(ql, BLOCK)
        F.pool_blocks(kl, BLOCK)
    ev[1].record(stream)
    for _ in range(reps):
        F.fft_block_mask(ql, kl, **kw)
    ev[2].record(stream)
    out_l = torch.empty(1, L, shard.heads, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    attn_status = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(reps):
        F.sparse_attention(ql, kl, vl, mask.bits, BLOCK, out=out_l, status=attn_status)
    ev[3].record(stream)
    torch.cuda.synchronize(dev)
    t_pool = ev[0].elapsed_time(ev[1]) / reps
    t_mask = ev[1].elapsed_time(ev[2]) / reps  # includes pooling
    t_attn = ev[2].elapsed_time(ev[3]) / reps
    if int(attn_status.item()) != 0:
        raise RuntimeError(f"attention kernel reported status {int(attn_status.item())} (a bounded wait timed out)")
    pairs = causal_pairs(mask.bits, L, BLOCK)
    flops = 4.0 * HEAD_DIM * pairs
    hbm_peak, bf16_peak, bf16_sustained, peak_kind = load_peaks()
    achieved = flops / (t_attn * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(HERE, "profiles", "attn_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                traffic = json.load(f).get("bytes_per_launch")
        except (OSError, ValueError, AttributeError):
            traffic = None
    roofline = {"kernel": "sparse_attn_kernel", "bound": "tensor", "achieved": round(achieved, 1),
                "peak": bf16_peak, "unit": "TFLOP/s", "frac": round(achieved / bf16_peak, 4),
                "peak_kind": f"{peak_kind} bf16 burst", "traffic": traffic,
                "peak_sustained": bf16_sustained, "frac_sustained": round(achieved / bf16_sustained, 4),
                "algorithmic_flops_per_launch": flops, "launch_ms": round(t_attn, 4),
                "causal_pair_density": pairs / (shard.heads * L * (L + 1) / 2)}
    pool_bytes = (ql.numel() + kl.numel()) * 2 + mask.q_pooled.numel() * 2 + mask.k_pooled.numel() * 2
    try:
        sel_kernels = kernel_times_us(lambda: F.fft_block_mask(ql, kl, pooled=(mask.q_pooled, mask.k_pooled), **kw))
    except Exception as exc:  # noqa: BLE001 - the activity trace is a report, not a requirement
        sel_kernels = {"error": f"{exc}"[:200]}
    # ---- N > 1: the fused gather's parts on every rank (its own heads' attention
    # without pushes, the same attention storing every tile to all peers, then the
    # flag store and the wait for the slowest peer)
    gather_parts = None
    if world > 1 and pg is not None:
        torch.cuda.synchronize(dev)
        barrier()
        tim = []
        for _ in range(reps):
            pg.run(ql, kl, vl, mask.bits, BLOCK, True, shard, timing=tim)
        torch.cuda.synchronize(dev)
        pg.check()
        t_push = sum(a.elapsed_time(b) for a, b, _ in tim) / reps
        t_wait = sum(b.elapsed_time(c) for _, b, c in tim) / reps
        mine = torch.tensor([t_attn, t_push, t_wait], device=dev)
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        every = torch.stack(every).cpu().tolist()
        gather_parts = {"attention_ms_per_rank": [round(r[0], 4) for r in every],
                        "attention_with_push_ms_per_rank": [round(r[1], 4) for r in every],
                        "flag_wait_ms_per_rank": [round(r[2], 4) for r in every]}
    stages = {"pool_ms": round(t_pool, 4), "pool_gbs": round(pool_bytes / (t_pool * 1e-3) / 1e9, 1),
              "pool_frac_hbm": round(pool_bytes / (t_pool * 1e-3) / 1e9 / hbm_peak, 4),
              "select_ms": round(t_mask - t_pool, 4), "select_kernels_us": sel_kernels,
              "attention_ms": round(t_attn, 4),
              "block_density": round(mask.density(), 5),
              "stripe_heads": int(mask.is_stripe.sum().item())}
    if gather_parts is not None:
        stages["gather_parts"] = gather_parts

    # ---- selection sweep: BASELINE config 3 sweeps keep ratios {0.02, 0.05, 0.1}, and
    # the reference's only published 128K number is threshold mode at T = 0.9.  The
    # same step at each setting, 3 timed steps after one untimed, max over ranks, with
    # the block density of this rank's heads.  A failure is reported in the field
    # instead of ending the run (every rank runs the same code, so all take the same path).
    sweep = {}
    for name, kwr in (("topk 0.02", mask_kwargs(0.02)), ("topk 0.05", mask_kwargs(0.05)),
                      ("topk 0.1", mask_kwargs(0.1)), ("threshold 0.9", threshold_kwargs(0.9))):

        def step_r():
            if world == 1:
                return F.myattn_prefill(q, k, v, 0, **kwr)
            return sharded_prefill(q, k, v, 0, num_kv_heads=HKV, gather=pg, **kwr)
        try:
            step_r()
            torch.cuda.synchronize(dev)
            barrier()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(3):
                step_r()
            s1.record(stream)
            torch.cuda.synchronize(dev)
            tr = torch.tensor([s0.elapsed_time(s1) / 3], device=dev)
            if world > 1:
                dist.all_reduce(tr, op=dist.ReduceOp.MAX)
            sweep[name] = {"ms_per_layer": round(float(tr.item()), 4),
                           "block_density": round(F.fft_block_mask(ql, kl, **kwr).density(), 5)}
        except Exception as exc:  # noqa: BLE001
            sweep[name] = {"error": f"{exc}"[:200]}

    # ---- the caller-side kernels (rope_pool, decode) against the HBM copy peak
    caller = None
    if not args.no_caller_kernels:
        try:
            caller = caller_side_kernels(dev, L, hbm_peak, bf16_peak)
        except Exception as exc:  # noqa: BLE001 - reported in the field instead of ending the run
            caller = {"error": f"{exc}"[:200]}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        qh, kh, vh = (x.cpu().pin_memory() for x in local_views(q, k, v, shard))
        res_h = torch.empty(1, shard.heads, L, HEAD_DIM, dtype=torch.bfloat16).pin_memory() if world > 1 else \
            torch.empty(1, L, HQ * HEAD_DIM, dtype=torch.bfloat16).pin_memory()
        del q, k, v
        torch.cuda.empty_cache()

        # N = 1: the drop-in operator on the whole layer, from pinned host buffers through
        # myattn_prefill_host (copies of one head chunk overlap the work on another).
        # N > 1: each rank receives
        # its own q/k/v heads, runs its shard with the peer-memory all-gather, and
        # reads back its own heads of the gathered output (all ranks together read
        # the whole output once).
        def e2e_step():
            if world == 1:  # head chunks copied in, computed and read back on three streams
                F.myattn_prefill_host(qh, kh, vh, 0, out=res_h, **kw)
                return
            qd = qh.to(dev, non_blocking=True)
            kd = kh.to(dev, non_blocking=True)
            vd = vh.to(dev, non_blocking=True)
            full = sharded_prefill(qd, kd, vd, 0, num_heads=HQ, num_kv_heads=HKV, inputs_are_local=True,
                                  gather=pg, **kw)
            res_h.copy_(full[:, shard.h_lo:shard.h_hi], non_blocking=True)

        e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e2.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        te = torch.tensor([s2.elapsed_time(e2) / args.e2e_steps], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": round(float(te.item()), 3), "unit": UNIT,
               "h2d_bytes_per_step": int((qh.numel() + kh.numel() + vh.numel()) * 2) * world,
               "d2h_bytes_per_step": int(res_h.numel() * 2) * world, "steps": args.e2e_steps,
               "bytes": "whole job (every rank copies its own heads)" if world > 1 else "one GPU"}

    ttft = None
    if not args.no_ttft:
        ttft = run_ttft(args, dev, world, rank, stream, barrier, pg)
    if pg is not None and int(pg.status.item()) != 0:
        raise RuntimeError("the peer-memory all-gather reported a wait time-out (a peer never delivered its rows)")
    torch.cuda.synchronize(dev)
    clocks.__exit__(None, None, None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from fftsparse_b200.synthetic import make_inputs as mk
        qc, kc, vc = mk(L, num_q_heads=HQ, num_kv_heads=HKV, dtype=torch.bfloat16)
        cms, info = cpu_baseline_sample(qc, kc, vc, args.keep_ratio)
        cpu = {"value": round(cms, 1), "unit": UNIT, "cores": info["threads"], "kind": "port",
               "sample": f"full {L}-token mask selection (C oracle, {info['cpu_count']} OpenMP threads) "
                         f"{info['mask_s']:.2f} s + fp32 attention for head 0 on {info['rows_sampled']} query "
                         f"blocks {info['attn_sample_s']:.2f} s scaled by kept blocks x{info['attn_scale']:.1f}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms_max, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms_max, 4), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg3: L={L}, Hq={HQ}, Hkv={HKV}, D={HEAD_DIM}, block {BLOCK}, keep ratio "
                                   f"{args.keep_ratio} (topk mode, efficiency-script ratios); "
                                   + ("drop-in myattn_prefill with repeat_kv-expanded k/v" if world == 1 else
                                      f"KV groups sharded {HKV // world} per rank; output all-gather fused into the "
                                      f"attention epilogue (peer stores over NVLink)"),
                       "model": "Llama-3.1-8B attention-layer shape", "seq_len": L, "global_batch": 1,
                       "parallelism": "single GPU" if world == 1 else f"kv-group x{world}",
                       "l2": "inputs (3.2 GB) larger than L2; no flush"},
            "clocks": clocks.summary(),
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "stages": stages,
            "gqa_native_ms_per_layer": round(gqa_native_ms, 4),
            "host_issue_ms_per_step": round(host_ms, 4),
            "selection_sweep": dict(sweep, note="threshold 0.9 uses the settings of the reference's published "
                                                "128K run (77.8 ms/layer on an unrecorded A100-class GPU with "
                                                "captured Llama-3.1-8B Q/K; here synthetic inputs, so block "
                                                "densities differ)"),
            "ttft": ttft,
            "caller_kernels": caller,
        }
        emit(line)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


# The JSON result line goes to the process's real stdout; everything else written
# to file descriptor 1 (library banners such as NCCL's version line included) is
# sent to stderr, so that stdout carries the result line alone.
_RESULT = None


def emit(line: dict) -> None:
    out = _RESULT if _RESULT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _RESULT
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse()
    if args.caller_kernels_only:
        import fftsparse_b200 as F
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        F.load_library()
        hbm_peak, bf16_peak, _, peak_kind = load_peaks()
        emit({"caller_kernels": caller_side_kernels(dev, args.seq_len, hbm_peak, bf16_peak, reps=args.steps),
              "seq_len": args.seq_len, "peak_kind": peak_kind})
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
