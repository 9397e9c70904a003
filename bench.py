"""Benchmark of the B200 hot path of wan-dit-lab's Wan-5B DiT block forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload rollout|linear]

Workload "rollout" (default): the full 30-layer Wan2.2-TI2V-5B-shaped DiT with random-init
W4A4 weights (N(0, 0.02), seed 6) generating a 512x928 video chunk by chunk: latent [48, 21, 32, 58] N(0,1)
noise (seed 8), a 512 x 4096 bf16 prompt N(0,1) (seed 9), chunks of 3 latent frames (1392 tokens), 4 DMD steps
+ 1 write pass per chunk, an FP8 KV window of 21 latent frames, 7 chunks. One step = one whole rollout of 21
latent frames; metric = latent frames / s (value summed over ranks: one independent stream per GPU). The W4A4
GEMMs (5 per block, 150 per pass) are timed with CUDA events in one extra instrumented chunk after the timed
region: their algorithmic int ops over their event time is the roofline figure.

Workload "linear" (the W4A4 QKV linear): X bf16 [1392, 3072] N(0,1) with 1% outlier
channels x20, W [9216, 3072] N(0, 0.02) quantized to INT4 groups of 64 with float16 scales; one step = one
w4a4 linear call (activation quantizer + tcgen05 GEMM) on inputs resident in HBM. Inputs are synthetic and
seeded (the reference publishes no dataset for this path).

Timing: W warm-up steps, then K timed steps. Every timed step is bracketed by CUDA events on the launching
stream; between steps (outside the events) a 512 MiB buffer is written to flush the 126 MB L2, so each step
starts cold (the rollout's 5 GB of weights exceed L2 anyway). Under torchrun every rank runs its own replica (this path shards into independent streams: no
collective on the data path); the time is the max over ranks, the value the sum of the ranks' work over it.

One JSON line (rank 0): metric/value/unit, e2e (the same call from pinned host buffers, copies included),
roofline of the GEMM kernel (algorithmic int ops / its CUDA-event time vs the measured INT8 peak), the CPU
baseline (the reference's own CPU torch path on the host cores, a bounded sample: ReferenceBlockPass), clocks
sampled by nvidia-smi while timing. `--impl reference` times that same reference path, one block pass per step (its
W4A4 and Sage kernels are third-party sm_89 CUDA that neither runs on a CPU nor ships in its tree; on a CPU the
reference runs its block with bf16 nn.Linear layers and exact attention over the FP8 cache). The reference package
is imported, unmodified, from baseline/_ref (baseline/install_reference.sh).
"""

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "wan-dit-lab_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "latent frames/s per GPU (5B DiT, 512x928) and W4A4 GEMM TOPS vs INT8 peak"
METRIC_LINEAR = "W4A4 GEMM TOPS vs INT8 peak"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
INT8_NOMINAL_TOPS = 4500.0
CODES = "f16pre"  # operand code format of the W4A4 GEMM (--codes)
GEMM_KERNEL = {"int8": "w4a4_gemm_kernel", "e4m3": "w4a4_gemm_kernel", "f16fold": "gemm_fold_kernel", "f16pre": "gemm_pre_kernel (FFN-2: gemm_fold_kernel)"}


def _measured_bf16_peak():
    try:
        return float(json.loads(PEAKS_FILE.read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return None


# DRAM traffic per GEMM launch from one ncu capture of a block pass (dram__bytes_read.sum + dram__bytes_write.sum,
# mean over its six launches); the capture and its command are in the profiles folder.
GEMM_TRAFFIC = {"f16fold": 76.3e6, "f16pre": 74.4e6}
GEMM_TRAFFIC_SOURCE = "profiles/gemm_pre_and_fold_kernels_block_pass_1392_tokens.md"

F16_PEAK_TFLOPS = _measured_bf16_peak()  # the folded format runs on the 16-bit tensor pipe: its own ceiling


def seeded(shape, seed, scale=1.0, outliers=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers:
        cols = torch.randperm(shape[-1], generator=g)[: max(1, int(outliers * shape[-1]))]
        x[..., cols] *= 20
    return x


class Clocks:
    """nvidia-smi sampled every 200 ms in a background process while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=lambda: self.lines.extend(self.proc.stdout), daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)
            self.reader.join(timeout=2)

    def summary(self):
        sm, sm_max, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                sm_max = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": sm_max,
                "reasons": sorted(reasons), "samples": len(sm)}


def int8_peak_tops(device):
    """Dense INT8 peak measured here: cuBLASLt int8 GEMM (torch._int_mm) 8192^3, best of 10. Falls back to 2x the
    measured bf16 peak of MEASURED_PEAKS.json (B200's dense INT8 rate is twice its BF16 rate)."""
    try:
        a = torch.randint(-8, 8, (8192, 8192), dtype=torch.int8, device=device)
        b = torch.randint(-8, 8, (8192, 8192), dtype=torch.int8, device=device).t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e) / 1e3)
        del a, b
        return 2 * 8192 ** 3 / best / 1e12, "measured here: cuBLASLt int8 GEMM (torch._int_mm) 8192^3, best of 10"
    except Exception as error:  # noqa: BLE001 - a missing int8 GEMM falls back to the documented ratio
        peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
        bf16 = peaks.get("bf16_tflops", 1590.0)
        return 2 * bf16, f"2 x bf16 peak of MEASURED_PEAKS.json ({type(error).__name__} measuring int8)"


def flush_l2(buf):
    buf.add_(1)


def timed_steps(run, steps, flush, stream):
    """Per-step CUDA-event times (seconds) of `run`, the L2 flushed before each step outside the events."""
    times = []
    for _ in range(steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        run()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e) / 1e3)
    return times


def linear_workload(device):
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.quantization import w4a4
    M, K, N = 1392, 3072, 9216
    x = seeded((M, K), 0, outliers=0.01).to(torch.bfloat16)
    W = seeded((N, K), 1, scale=0.02)
    parts = w4a4.quantize(W.to(device), rank=0, scale_dtype=torch.float16)
    layer = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=CODES)
    xd = x.to(device)
    lib = _native.lib()
    work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device=device)
    codes = work[: M * K * 2]  # the activation codes the quantizer left in the workspace (one or two bytes each)
    scales = work[(M * K * 2 + 255) // 256 * 256:].view(torch.float32)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=device)
    st = _native.stream(device)

    fmt = layer.code_format

    def step():  # the public entry point: quantizer + GEMM (2 kernels)
        _native.check(lib.wdl_w4a4_linear(xd.data_ptr(), K, M, K, None, _native.F16, layer.codes.data_ptr(),
                                          layer.scales.data_ptr(), fmt, None, N, y.data_ptr(), N, work.data_ptr(),
                                          work.numel(), st))

    def gemm_only():  # the dominant kernel alone, on the activation codes the quantizer left in the workspace
        _native.check(lib.wdl_w4a4_gemm(codes.data_ptr(), scales.data_ptr(), layer.codes.data_ptr(),
                                         layer.scales.data_ptr(), fmt, None, M, N, K, y.data_ptr(), N, st))

    x_host = x.pin_memory()
    y_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()

    def e2e_step():  # host -> device copy of X, the call, device -> host copy of Y
        xd.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y, non_blocking=True)

    ops = 2 * M * N * K
    return dict(step=step, kernel=gemm_only, e2e=e2e_step, ops=ops, launches_per_step=2,
                h2d=x.numel() * 2, d2h=M * N * 2,
                config={"workload": "BASELINE config 1: W4A4 QKV linear X[1392,3072] x W[9216,3072]^T",
                        "M": M, "N": N, "K": K, "group": 64, "scale_dtype": "float16", "codes": CODES,
                        "l2": "flushed between steps"},
                algorithmic={"int_ops_per_launch": ops, "bytes_per_launch": M * K + N * K + M * N * 2 + (K // 64) * (M + N) * 4},
                cpu=lambda: cpu_linear_sample(x, W), dtype="int4 x int4 -> int32 (int8 tensor cores), fp32 promote")


def cpu_linear_sample(x, W, repeats=3):
    """The reference's CPU torch path for this layer: its nn.Linear in bf16 (as its torch block runs q, k, v under
    bf16 autocast; W4A4 itself has no CPU path in the reference), at full size, all host threads. Returns (seconds
    per call, int ops, sample description)."""
    torch.set_num_threads(os.cpu_count())
    xb, Wb = x.to(torch.bfloat16), W.to(torch.bfloat16)
    torch.nn.functional.linear(xb, Wb)
    t0 = time.perf_counter()
    for _ in range(repeats):
        torch.nn.functional.linear(xb, Wb)
    dt = (time.perf_counter() - t0) / repeats
    return dt, 2 * x.shape[0] * W.shape[0] * W.shape[1], (
        f"torch.nn.functional.linear in bf16 (the reference's nn.Linear) [1392,3072]x[9216,3072]^T at full size, "
        f"{torch.get_num_threads()} threads, mean of {repeats} calls")


def rollout_workload(device, rank=0, chunks=7, layers=30, tp=None, graphs=True, height=512, width=928, svd_rank=0):
    """tp = (world, reduce): one stream split across the ranks (tensor parallelism), else one stream per rank.
    height x width pixels: 512 x 928 (464 tokens a frame) or 704 x 1280 (config 5, 880).
    svd_rank: every layer's SVDQuant low-rank branch (0: none, BASELINE's configs; 32: the LongLive packs')."""
    from wan_dit_lab_b200.generation import causal
    from wan_dit_lab_b200.models.block import WanBlockB200
    from wan_dit_lab_b200.models.block_tp import WanBlockTP
    from wan_dit_lab_b200.quantization import w4a4
    w4a4.CODE_FORMAT = CODES  # every block's layers in the --codes operand format
    torch.manual_seed(0)
    world = 1 if tp is None else tp[0]
    model = causal.random_model(seed=6, device=device, num_layers=layers,
                                shard=None if tp is None else (rank, world), reduce=None if tp is None else tp[1],
                                svd_rank=svd_rank)
    block_cls = WanBlockB200 if tp is None else WanBlockTP
    seed_rank = rank if tp is None else 0  # the ranks of a split stream share its noise
    g = torch.Generator().manual_seed(8 + 1000 * seed_rank)  # one independent seeded stream per rank
    lat_h, lat_w = height // 16, width // 16  # the VAE's stride 16
    tokens = 3 * (lat_h // 2) * (lat_w // 2)  # a chunk of 3 latent frames, 2 x 2 patches
    noise = torch.randn(48, 21, lat_h, lat_w, generator=g)
    text = torch.randn(1, 512, 4096, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    stream = causal.Stream(model, text.to(device), height, width,
                           torch.Generator(device=device).manual_seed(10 + seed_rank), vae_stride=16,
                           cuda_graph=graphs)  # passes replayed from CUDA graphs (a split's all-reduces with them)
    noise_d = noise.to(device)
    out = torch.empty_like(noise_d)

    def step():
        stream.reset()
        for c in range(chunks):
            out[:, 3 * c:3 * c + 3] = stream.next_chunk(noise_d[:, 3 * c:3 * c + 3])

    noise_host = noise.pin_memory()
    out_host = torch.empty_like(noise).pin_memory()

    def e2e_step():
        noise_d.copy_(noise_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)

    gemm_log = []

    def gemm_only():
        """One instrumented chunk: the W4A4 GEMM launches bracketed by CUDA events (returns seconds, ops)."""
        gemm_log.clear()
        block_cls.gemm_timer = lambda e0, e1, ops: gemm_log.append((e0, e1, ops))
        graphed, stream.use_graphs = stream.use_graphs, False  # launched eagerly, so that each GEMM can be timed
        try:
            stream.reset()
            stream.next_chunk(noise_d[:, :3])
        finally:
            block_cls.gemm_timer = None
            stream.use_graphs = graphed
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b, _ in gemm_log) / 1e3, sum(o for _, _, o in gemm_log), len(gemm_log)

    per_block = 2 * tokens * 3072 * (9216 + 3072 + 3072 + 3072 + 2 * 14336) // world  # this rank's share
    window = 21 * tokens // 3  # keys of the 21-frame window
    config5 = (height, width) == (704, 1280)
    name = ("BASELINE config 5: 30-layer 5B DiT rollout, 704x1280 (880 tokens a frame, 2640-token chunks, up to 18480 "
            "keys), 7 chunks x (4 DMD steps + write pass), FP8 KV window 21 frames" if config5 else
            "BASELINE config 4: 30-layer 5B DiT rollout, 512x928, 7 chunks x (4 DMD steps + write pass), FP8 KV window "
            "21 frames" if (height, width) == (512, 928) else
            f"30-layer 5B DiT rollout, {height}x{width}, 7 chunks x (4 DMD steps + write pass), FP8 KV window 21 frames")
    # kernels per block: 20 (5 for Sage attention over the cache), 25 with the split (rows_sumsq x 2, the sharded
    # norms in place of the fused ones, residual_update x 3); + 1 modulation launch per pass
    return dict(step=step, e2e=e2e_step, gemm_probe=gemm_only, frames=3 * chunks,
                launches_per_step=chunks * 5 * (1 + layers * (20 if tp is None else 25)),
                h2d=noise.numel() * 4, d2h=noise.numel() * 4,
                config={"workload": name,
                        "model": "Wan2.2-TI2V-5B shape, random init N(0,0.02), W4A4 (INT4 g64, bf16 scales, "
                                 f"SVD rank {svd_rank})",
                        "tokens_per_chunk": tokens, "keys_per_chunk": [min(tokens * (c + 1), window) for c in range(chunks)],
                        "chunks": chunks, "layers": layers, **({} if tp is None else {"tensor_parallel": world}),
                        "cuda_graphs": bool(graphs),
                        "codes": CODES, "l2": "inputs larger than L2 (5 GB of weights per pass)"},
                algorithmic={"gemm_int_ops_per_block_pass": per_block, "gemm_launches_per_block_pass": 6},
                cpu=lambda: cpu_block_sample(tokens=tokens, grid=(3, lat_h // 2, lat_w // 2)), dtype="W4A4 (int4 x int4 exact on int8 tensor cores) + INT8/FP8 Sage "
                                                      "attention; fp32 residual stream")


REF_PACKAGE = ROOT / "baseline" / "_ref"
BLOCK_PASSES_PER_ROLLOUT = 30 * 7 * 5  # 30 blocks x 7 chunks x (4 denoising passes + the write pass)


class ReferenceBlockPass:
    """One pass of the reference's own Wan block on the host CPU, as its rollout runs it (reference
    generation/causal.py Pass.run: the block under bf16 autocast; models/block.py WanBlock with nn.Linear layers,
    models/multi_head_attention.py, KVCache(fp8=True).attend, which on a CPU stores the chunk in FP8 and attends
    with exact SDPA over the cache read back to bf16). The reference package, unmodified, is imported from
    baseline/_ref (baseline/install_reference.sh). Shapes of BASELINE config 3 inside the config-4 rollout: dim 3072,
    24 heads, FFN 14336, a 1392-token chunk of 3 frames (16 x 29) over 4176 cached keys of 9 frames (the mean
    cache fill before the 7 chunks of the rollout: 0, 1392, ... 8352 keys) and a 512-token prompt whose keys and
    values are computed once (context_kv, as the reference's Stream caches them per prompt). Weights N(0, 0.02);
    the linears in bf16, the norms and the modulation in float32 (a CPU layer_norm takes float32 parameters only).
    Calling it times one pass (seconds); each pass writes the chunk at the same place, so passes repeat exactly."""

    def __init__(self, tokens=1392, cached=None, text=512, seed=11, grid=(3, 16, 29)):
        if not (REF_PACKAGE / "wan_dit_lab").is_dir():
            raise RuntimeError(f"the reference package is not installed in {REF_PACKAGE}: run "
                               "baseline/install_reference.sh")
        if str(REF_PACKAGE) not in sys.path:
            sys.path.insert(0, str(REF_PACKAGE))
        from wan_dit_lab.generation.causal import KVCache
        from wan_dit_lab.models.block import WanBlock
        from wan_dit_lab.models.rope import rope
        torch.set_num_threads(os.cpu_count())
        dim, ffn, heads = 3072, 14336, 24
        per_frame = grid[1] * grid[2]
        if cached is None:  # the mean cache fill before the 7 chunks: 0, 1, ... 6 chunks of keys
            cached = 3 * tokens
        g = torch.Generator().manual_seed(seed)
        blk = WanBlock(dim, ffn, heads, 1e-6)
        with torch.no_grad():
            for name, p in blk.named_parameters():
                if name == "modulation":
                    p.copy_(torch.randn(p.shape, generator=g) / dim ** 0.5)
                elif "norm" in name:
                    p.fill_(1.0 if name.endswith("weight") else 0.0)
                else:
                    p.copy_(torch.randn(p.shape, generator=g) * 0.02)
        for module in blk.modules():
            if isinstance(module, torch.nn.Linear):
                module.to(torch.bfloat16)
        self.block = blk.eval()
        d = 128  # the Live preset's float32 table: time / height / width pairs 22 / 21 / 21
        self.freqs = torch.cat([rope(1024, d - 4 * (d // 6)), rope(1024, 2 * (d // 6)), rope(1024, 2 * (d // 6))],
                               dim=-1).float()
        self.grid = (tuple(grid),)
        self.cache = KVCache(18 * per_frame, fp8=True, chunk=3)  # a window of 21 frames less the chunk
        self.X = torch.randn(1, tokens, dim, generator=g)  # the float32 stream of blocks after the first
        self.e0 = torch.randn(1, 6, dim, generator=g) * 0.1
        context = torch.randn(1, text, dim, generator=g).to(torch.bfloat16)
        with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
            self.context_kv = blk.cross_attn.keys_values(context)
            self.cache.allocate(torch.empty(1, tokens, heads, d, dtype=torch.bfloat16))
            self.cache.store(0, torch.randn(1, cached, heads, d, generator=g), torch.randn(1, cached, heads, d, generator=g))
        self.cache.saved, self.cache.frames = cached, cached // per_frame
        self.threads = torch.get_num_threads()
        self.sample = (f"the reference's own WanBlock (bf16 nn.Linear under autocast) + KVCache(fp8=True).attend (exact "
                       f"SDPA over the FP8 cache) on the host CPU, {self.threads} threads: one block pass of {tokens} "
                       f"tokens over {cached} cached keys and a {text}-token prompt, x {BLOCK_PASSES_PER_ROLLOUT} "
                       "block passes (30 blocks x 35 passes) per 21-frame rollout")

    @torch.no_grad()
    def __call__(self):
        with torch.autocast("cpu", dtype=torch.bfloat16):
            t0 = time.perf_counter()
            self.block(self.X, self.e0, grid_sizes=self.grid, freqs=self.freqs, context_kv=self.context_kv,
                       start_frame=0, cache=self.cache)
            return time.perf_counter() - t0


def cpu_block_sample(passes=3, tokens=1392, grid=(3, 16, 29)):
    """The CPU baseline of the rollout: the median of `passes` timed reference block passes (after one untimed),
    extrapolated by block passes only. Returns (seconds per rollout, frames, sample description)."""
    ref = ReferenceBlockPass(tokens=tokens, grid=grid)
    ref()
    per_pass = statistics.median(ref() for _ in range(passes))
    return per_pass * BLOCK_PASSES_PER_ROLLOUT, 21, ref.sample + f"; median of {passes} passes"


WORKLOADS = {"rollout": rollout_workload, "linear": linear_workload}


def combine_ranks(dist, seconds, device):
    """Max over ranks of each of the per-rank durations `seconds` (every rank calls this, in the same order)."""
    t = torch.tensor(seconds, device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_rate(world, units_per_rank, seconds_max):
    """Whole-job throughput: every rank processes units_per_rank; the job lasts as long as its slowest rank."""
    return world * units_per_rank / seconds_max


def reference_arm(args, rank, world):
    """The reference's own CPU torch path on the host cores, on rank 0 only (the other ranks exit): each step one
    reference block pass (rollout: value = 21 latent frames over the pass time x 1050 block passes per rollout) or
    one full-size bf16 nn.Linear call (linear: TOPS)."""
    if rank != 0:
        return
    times = []
    if args.workload == "rollout":
        try:
            ref = ReferenceBlockPass()
        except (RuntimeError, ImportError) as error:  # the reference package is not installed here
            print(json.dumps({"impl": "reference", "unavailable": str(error).splitlines()[0]}), flush=True)
            return
        for _ in range(args.warmup):
            ref()
        times = [ref() for _ in range(args.steps)]
        t = statistics.mean(times)
        value, unit, metric = 21 / (t * BLOCK_PASSES_PER_ROLLOUT), "latent frames/s", METRIC
        sample = ref.sample
        config = {"workload": "BASELINE config 4: 30-layer 5B DiT rollout, 512x928, 7 chunks x (4 DMD steps + write pass), "
                              "FP8 KV window 21 frames", "step": "one reference block pass (BASELINE config 3 shapes, "
                              "4176 cached keys); value extrapolates x 30 blocks x 35 passes", "threads": ref.threads}
        dtype = "bf16 (the reference's nn.Linear under autocast), FP8 KV cache, exact SDPA"
    else:
        x = seeded((1392, 3072), 0, outliers=0.01).to(torch.bfloat16)
        W = seeded((9216, 3072), 1, scale=0.02)
        for _ in range(args.warmup):
            cpu_linear_sample(x, W, repeats=1)
        for _ in range(args.steps):
            dt, ops, sample = cpu_linear_sample(x, W, repeats=1)
            times.append(dt)
        t = statistics.mean(times)
        value, unit, metric = ops / t / 1e12, "TOPS", METRIC_LINEAR
        config = {"workload": "BASELINE config 1: W4A4 QKV linear X[1392,3072] x W[9216,3072]^T (bf16 nn.Linear on "
                              "the CPU: the reference has no CPU W4A4 path)"}
        dtype = "bf16"
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded, BASELINE shapes)",
            "config": config,
            "cpu_baseline": {"value": value, "unit": unit, "cores": torch.get_num_threads(), "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None, help="timed steps (default 5 rollouts / 20 linears)")
    parser.add_argument("--warmup", type=int, default=None, help="warm-up steps (>= 3)")
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--workload", default="rollout", choices=sorted(WORKLOADS))
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    parser.add_argument("--codes", default="f16pre", choices=("e4m3", "f16fold", "f16pre", "int8"),
                        help="operand code format of the W4A4 GEMM: e4m3 (kind::f8f6f4), f16fold (float16 codes and scale-folded weights, "
                             "kind::f16), f16pre (f16fold with the activation scales folded in too: all of K "
                             "accumulated on the tensor cores) or int8 (kind::i8)")
    parser.add_argument("--chunks", type=int, default=7, help="rollout chunks (profiling; BASELINE config 4: 7)")
    parser.add_argument("--layers", type=int, default=30, help="model layers (profiling; BASELINE config 4: 30)")
    parser.add_argument("--eager", action="store_true", help="launch every kernel from Python (no CUDA graphs)")
    parser.add_argument("--height", type=int, default=512, help="pixels (BASELINE config 4: 512; config 5: 704)")
    parser.add_argument("--width", type=int, default=928, help="pixels (BASELINE config 4: 928; config 5: 1280)")
    parser.add_argument("--tp", action="store_true",
                        help="BASELINE config 5b: one stream split across the ranks (heads / hidden channels, NCCL "
                             "all-reduce after O, cross-O and FFN-2) instead of one independent stream per rank")
    parser.add_argument("--svd-rank", type=int, default=0,
                        help="rank of every layer's SVDQuant low-rank branch (BASELINE's configs: 0; the LongLive "
                             "W4A4 packs: 32)")
    args = parser.parse_args()
    global CODES
    CODES = args.codes
    rollout = args.workload == "rollout"
    if args.steps is None:
        args.steps = 5 if rollout else 20
    if args.warmup is None:
        args.warmup = 3 if rollout else 5
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    args.warmup = max(args.warmup, 3)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    if args.tp and not rollout:
        parser.error("--tp splits the rollout")
    tp = (world, (lambda t: dist.all_reduce(t)) if dist is not None else (lambda t: None)) if args.tp else None
    wl = (WORKLOADS[args.workload](device, rank, args.chunks, args.layers, tp, not args.eager, args.height, args.width,
                                   args.svd_rank)
          if rollout else WORKLOADS[args.workload](device))
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    flush = lambda: flush_l2(flush_buf)  # noqa: E731

    for _ in range(args.warmup):
        wl["step"]()
    torch.cuda.synchronize()
    peak, peak_source = int8_peak_tops(device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # the timed region: K steps through the public API, inputs resident in HBM
    barrier()
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed region (ncu --nvtx-include timed/)
    with Clocks(local) as clocks:
        times = timed_steps(wl["step"], args.steps, flush, stream)
    torch.cuda.nvtx.range_pop()
    barrier()
    step_s = sum(times) / len(times)
    # end to end from pinned host buffers (host <-> device copies inside the timed region)
    for _ in range(2 if not rollout else 1):
        wl["e2e"]()
    e2e_times = timed_steps(wl["e2e"], args.steps, flush, stream)
    e2e_s = sum(e2e_times) / len(e2e_times)
    # the dominant kernel
    if rollout:
        gemm_s, gemm_ops, gemm_launches = wl["gemm_probe"]()
        achieved = gemm_ops / gemm_s / 1e12
        kernel_ms = gemm_s / gemm_launches * 1e3
    else:
        kernel_times = timed_steps(wl["kernel"], args.steps, flush, stream)
        kernel_s = sum(kernel_times) / len(kernel_times)
        achieved, kernel_ms, gemm_launches = wl["ops"] / kernel_s / 1e12, kernel_s * 1e3, 1

    step_max, e2e_max = combine_ranks(dist, [step_s, e2e_s], device)
    streams = 1 if args.tp else world  # a split stream is one unit of work on all ranks (strong scaling)
    if rollout:
        value, e2e_value = job_rate(streams, wl["frames"], step_max), job_rate(streams, wl["frames"], e2e_max)
        unit, metric = "latent frames/s", METRIC
    else:
        value, e2e_value = job_rate(world, wl["ops"], step_max) / 1e12, job_rate(world, wl["ops"], e2e_max) / 1e12
        unit, metric = "TOPS", METRIC_LINEAR

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:  # the host baseline is taken at N = 1 only
        if rollout:
            try:
                per_rollout, frames, sample = wl["cpu"]()
                cpu = {"value": frames / per_rollout, "unit": unit, "cores": torch.get_num_threads(),
                       "kind": "reference", "sample": sample}
            except (RuntimeError, ImportError) as error:  # the reference package is not installed here
                print(f"cpu baseline unavailable: {error}", file=sys.stderr, flush=True)
        else:
            dt, cpu_ops, sample = wl["cpu"]()
            cpu = {"value": cpu_ops / dt / 1e12, "unit": "TOPS", "cores": torch.get_num_threads(), "kind": "reference",
                   "sample": sample}

    if rank == 0:
        dtype = wl["dtype"].replace("int8 tensor cores", {
            "int8": "int8 tensor cores (kind::i8)",
            "e4m3": "e4m3-coded integers on fp8 tensor cores (kind::f8f6f4), exact",
            "f16fold": "f16 tensor cores (kind::f16): int4 codes x int4 weights folded with their bf16 group scales, exact",
            "f16pre": "f16 tensor cores (kind::f16): int4 codes x bf16 scales on both operands (exact operands), "
                      "all of K accumulated in fp32 TMEM"}[CODES])
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_max * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.tp else "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded, BASELINE shapes)",
            "config": {**wl["config"], "parallelism": (f"tp{world}" if args.tp else f"streams{world}") if world > 1
                       else "single"},
            "e2e": {"value": e2e_value, "unit": unit, "ms_per_step": e2e_max * 1e3,
                    "h2d_bytes_per_step": wl["h2d"], "d2h_bytes_per_step": wl["d2h"]},
            "gpu_launches": wl["launches_per_step"] * args.steps,
            "roofline": {"bound": "tensor", "kernel": GEMM_KERNEL[CODES], "achieved": achieved, "peak": peak,
                         "unit": "TOPS", "frac": achieved / peak, "peak_source": peak_source,
                         "frac_of_measured_bf16_peak": achieved / F16_PEAK_TFLOPS if F16_PEAK_TFLOPS else None,
                         "frac_of_nominal_int8": achieved / INT8_NOMINAL_TOPS, "kernel_ms": kernel_ms,
                         "launches_measured": gemm_launches, "algorithmic": wl["algorithmic"],
                         "traffic": GEMM_TRAFFIC.get(CODES) if rollout and not args.tp else None,
                         "traffic_unit": "DRAM bytes read + written per GEMM launch (mean of a block pass's six)",
                         "traffic_source": GEMM_TRAFFIC_SOURCE if rollout and not args.tp and CODES in GEMM_TRAFFIC
                         else None},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        wl.clear()  # the passes' CUDA graphs (a split's hold NCCL calls) released before the process group
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
