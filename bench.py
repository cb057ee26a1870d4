"""Decode benchmark: Qwen3.5-9B-shaped W4A16 model, batch 1, on B200.

Workload (config 2 of the benchmark definition): a seeded random-init 32-layer package
(3:1 Gated-DeltaNet : full attention, vocab 248320, W4A16 g64, bf16 embeddings restricted
to fp16-representable values), a 512-token prefill of uniform random ids, then greedy
decode steps. A "step" is one decode token. `value` is decode tok/s over the timed steps
with everything resident in HBM (device time from CUDA events on the session stream);
`e2e` is the same metric through xq_decode_one (host call, token copied back every step).
`roofline` describes the dominant kernel, the persistent decode-step kernel (one launch per
token); `gemv_kernel` the standalone W4A16 GEMV of the per-op path.
With --gpus N (torchrun) every rank runs an independent replica session on its own GPU
(the path does not shard for replicas); value = all ranks' tokens / max rank time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__  # noqa: E402

PROMPT_LEN = 512
SEED = 2024
METRIC = "decode tok/s (9B W4A16, b=1)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def bf16_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def package_dir(preset="cfg2"):
    base = os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench"))
    return os.path.join(base, f"qwen35_9b_s{SEED}" if preset == "cfg2" else f"qwen35_{preset}_s{SEED}")


def make_package(rank, world, preset="cfg2"):
    from xqwen35_b200.packer import synthetic

    d = package_dir(preset)
    if rank == 0:
        t = time.time()
        synthetic.make_package(d, synthetic.preset(preset), seed=SEED)
        print(f"[bench] package ready in {time.time() - t:.1f}s: {d}", file=sys.stderr, flush=True)
    return d


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [float(s[1]) for s in self.samples if len(s) >= 9 and s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if len(s) >= 9 and s[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            if len(s) >= 9:
                for n, v in zip(names, s[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def ncu_traffic(kernel):
    """DRAM read + write bytes per launch of `kernel` from one ncu capture, kept as a figure in
    profiles/ncu_traffic.json (the capture command is recorded beside it); None if absent."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            e = json.load(f).get(kernel)
        return {"bytes": e["traffic_bytes_per_launch"], "source": e["source"]} if e else None
    except Exception:
        return None


def host_cpu():
    """The host's CPU model and core count, recorded next to every CPU-timed number."""
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count()}


def step_roofline(alg_bytes, ms_per_step, peak_gbs):
    """The dominant kernel is the persistent decode-step kernel (one launch per token, every
    phase of the step inside it). achieved = algorithmic bytes of one step / the mean launch
    duration from CUDA events on the session stream over the timed region."""
    achieved = alg_bytes / (ms_per_step * 1e-3) / 1e9
    tr = ncu_traffic("decode_step_kernel")
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": tr["bytes"] if tr else None,
            "traffic_source": tr["source"] if tr else None,
            "kernel": "decode_step_kernel", "algorithmic_bytes": int(alg_bytes),
            "launch_us": round(ms_per_step * 1000, 2)}


def gemv_roofline(pkg, peak_gbs, iters=40, engine="dp4a", rows=24576, cols=4096, max_copies=4):
    """A standalone W4A16 GEMV kernel of the kernel-level C ABI, timed with CUDA events on the
    launching stream: engine "dp4a" (gemv_w4a16_kernel, also the per-op path) or "mma" (the
    tensor-core gemv_mma_kernel, xqk_gemv_w4a16_mma). The default shape is the largest
    per-layer matrix of the 9B step (gate+up: 24576 x 4096), rotating over copies that together
    exceed L2; the lm_head shape (248320 x 4096, 540 MB) needs one copy."""
    import torch

    one = rows * cols // 2 + rows * (cols // 64) * 2
    ncopy = max(1, min(max_copies, -(-200_000_000 // one)))
    mats = []
    for i in range(ncopy):
        rng = np.random.default_rng(100 + i)
        packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
        s = (np.abs(rng.standard_normal(rows * cols // 64)) * 0.02).astype(np.float16).astype(np.float32)
        mats.append(pkg.Matrix(packed, s, np.full(rows * cols // 64, 8.0, np.float32), rows, cols, 64))
    x = torch.randn(cols, device="cuda")
    y = torch.zeros(rows, device="cuda")
    st = torch.cuda.current_stream()

    def run(m):
        (m.gemv_mma if engine == "mma" else m.gemv)(x.data_ptr(), y.data_ptr(), st.cuda_stream)

    for m in mats:
        run(m)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(iters):
        run(mats[i % ncopy])
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    alg = one + 4 * cols + 4 * rows
    achieved = alg / (ms * 1e-3) / 1e9
    for m in mats:
        m.close()
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4),
            "kernel": "gemv_mma_kernel" if engine == "mma" else "gemv_w4a16_kernel",
            "shape": f"{rows}x{cols}", "algorithmic_bytes": alg, "launch_us": round(ms * 1000, 2)}


def gemv_fixed_cost(pkg, peak_gbs):
    """Where a standalone tensor-core GEMV (xqk_gemv_w4a16_mma) spends the time its bytes do not
    explain: the same kernel at three row counts (K = 4096), each rotating over weight copies
    that together exceed L2, a least-squares fit of launch time = fixed + bytes / rate, and, as
    the floor of back-to-back launches on this stream, a one-element torch kernel timed the same
    way."""
    import torch

    pts = []
    for rows in (2368, 24576, 248320):  # 2368 = 148 blocks x 16 rows: one tile per block
        r = gemv_roofline(pkg, peak_gbs, iters=80, engine="mma", rows=rows, max_copies=48)
        pts.append((r["algorithmic_bytes"], r["launch_us"]))
    a = np.array([[1.0, b / 1e9] for b, _ in pts])
    fixed, per_gb = np.linalg.lstsq(a, np.array([t for _, t in pts]), rcond=None)[0]
    z = torch.zeros(1, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(10):
        z.add_(1.0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(200):
        z.add_(1.0)
    e1.record(st)
    torch.cuda.synchronize()
    empty_us = e0.elapsed_time(e1) * 1000 / 200
    return {"kernel": "gemv_mma_kernel", "cols": 4096,
            "points": [{"algorithmic_bytes": b, "launch_us": t} for b, t in pts],
            "fit_fixed_us": round(float(fixed), 2), "fit_stream_gb_s": round(1e6 / float(per_gb), 1),
            "empty_launch_us": round(empty_us, 2),
            "note": "launch time = fixed + bytes / stream rate over 2368, 24576 and 248320 rows; "
                    "empty_launch_us: back-to-back one-element kernels on the same stream"}


def config0_gemv(pkg, peak_gbs, iters=200):
    """Config 0 as specified: one W4A16 g64 GEMV, W [12288 x 4096] symmetric int4, x fp16
    ~ N(0, 1), y fp16, fp32 accumulation, through xqk_gemv_w4a16_mma_f16. Launched back to back
    over 8 weight copies (214 MB > L2), as a GEMV chain in a stream runs: each launch streams
    its own copy from HBM. Algorithmic bytes N*K/2 + N*(K/64)*2 + 2K + 2N = 26,771,456 per call.
    e2e: the same call with x in pinned host memory copied in and y copied out every call."""
    import torch

    rows, cols = 12288, 4096
    ncopy = 8
    mats = []
    for i in range(ncopy):
        rng = np.random.default_rng(300 + i)
        packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
        sc = (np.abs(rng.standard_normal(rows * cols // 64)) * 0.02).astype(np.float16).astype(np.float32)
        mats.append(pkg.Matrix(packed, sc, np.full(rows * cols // 64, 8.0, np.float32), rows, cols, 64))
    x = torch.randn(cols, device="cuda").half()
    y = torch.zeros(rows, device="cuda", dtype=torch.float16)
    st = torch.cuda.current_stream()
    for m in mats:
        m.gemv_mma_f16(x.data_ptr(), y.data_ptr(), st.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(iters):
        mats[i % ncopy].gemv_mma_f16(x.data_ptr(), y.data_ptr(), st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / iters * 1000
    alg = rows * cols // 2 + rows * (cols // 64) * 2 + 2 * cols + 2 * rows
    achieved = alg / (us * 1e-6) / 1e9
    # e2e through the kernel ABI with host buffers: pinned x in, y out, every call
    xh = torch.randn(cols).half().pin_memory()
    yh = torch.zeros(rows, dtype=torch.float16).pin_memory()
    n_e2e = 100
    for i in range(3):
        x.copy_(xh, non_blocking=True)
        mats[i % ncopy].gemv_mma_f16(x.data_ptr(), y.data_ptr(), st.cuda_stream)
        yh.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        x.copy_(xh, non_blocking=True)
        mats[i % ncopy].gemv_mma_f16(x.data_ptr(), y.data_ptr(), st.cuda_stream)
        yh.copy_(y, non_blocking=True)
        st.synchronize()
    e2e_us = (time.perf_counter() - t0) / n_e2e * 1e6
    for m in mats:
        m.close()
    return {"workload": "config0: W4A16 g64 GEMV 12288x4096, x/y fp16, fp32 accumulate, batch 1",
            "kernel": "gemv_mma_kernel<half, half>", "metric": "GEMV HBM GB/s", "value": round(achieved, 1),
            "unit": "GB/s", "us_per_call": round(us, 3), "algorithmic_bytes": alg,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved / peak_gbs, 4)},
            "l2": "8 weight copies (214 MB) rotated, each launch reads its copy from HBM",
            "launch": "back to back, programmatic dependent launch",
            "e2e": {"us_per_call": round(e2e_us, 2), "h2d_bytes_per_call": 2 * cols, "d2h_bytes_per_call": 2 * rows,
                    "api": "xqk_gemv_w4a16_mma_f16 with pinned host x / y copied every call"}}


def config1_step(pkg, peak_gbs, kv_fp16, steps=64):
    """Config 1: one decode step through two random-init 9B-shaped layers (DeltaNet + full
    attention) with the KV cache at 512 tokens: a 512-token prefill, then `steps` timed greedy
    steps (persistent step kernel, CUDA events on the session stream). The 234 MB of weights
    exceed L2. Algorithmic bytes per step: both layers' matrices and the lm_head (codes + fp16
    scales), the DeltaNet recurrent and conv states read and written, the KV cache read at the
    mean timed context and one row written, the embedding row."""
    d = package_dir("cfg1")
    from xqwen35_b200.packer import synthetic

    synthetic.make_package(d, synthetic.preset("cfg1"), seed=SEED)
    s = pkg.Session(d, device=0, kv_fp16=kv_fp16, max_context_tokens=512 + steps + 64)
    ids = np.random.default_rng(SEED + 1).integers(0, 1024, 512).astype(np.int32)
    s.prefill(ids)
    s.decode_timed(4)
    ms, _ = s.decode_timed(steps)
    info = json.loads(s.json("backend"))
    s.close()
    us = ms / steps * 1000
    kv_elem = 2 if kv_fp16 else 4
    ctx = 512 + 4 + steps / 2
    alg = (info.get("weight_bytes", 0) + 2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4 +
           2 * 4 * 256 * kv_elem * (ctx + 1) + 4096 * 2)
    achieved = alg / (us * 1e-6) / 1e9
    return {"workload": "config1: 2 layers (Gated-DeltaNet + GQA) at 9B shapes, vocab 1024, KV cache 512",
            "kernel": "decode_step_kernel", "us_per_step": round(us, 2), "algorithmic_bytes": int(alg),
            "kv_dtype": "f16" if kv_fp16 else "f32",
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved / peak_gbs, 4)},
            "l2": "inputs larger than L2 (234 MB of weights streamed per step)"}


def config3_sweep(pkg, peak_tflops, iters=5, split=False, shapes=None, m_values=(512, 2048, 8192)):
    """Config 3: the prefill W4A16 GEMM on tcgen05 / TMEM (xqk_prefill_gemm_w4a16) at M = 512,
    2048, 8192 tokens over 4096->12288, 12288->4096 and 4096->248320: bf16 activations ~ N(0, 1),
    symmetric int4 weights (scales ~ |N(0, 0.02)| in fp16), int4 dequantised to bf16 in shared
    memory, fp32 accumulation in tensor memory, bf16 output. TFLOP/s = 2 M N K / CUDA-event time
    (mean of `iters` launches after one warm-up) against the measured dense bf16 peak. With
    split=True: the split-bf16 mode (three products, the batched prefill's default)."""
    import torch

    out = []
    for (K, N) in shapes or ((4096, 12288), (12288, 4096), (4096, 248320)):
        rng = np.random.default_rng(K + N)
        packed = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
        sc = (np.abs(rng.standard_normal(N * K // 64)) * 0.02).astype(np.float16).astype(np.float32)
        m = pkg.Matrix(packed, sc, np.full(N * K // 64, 8.0, np.float32), N, K, 64)
        del packed, sc
        for M in m_values:
            x = torch.randn((M, K), device="cuda").to(torch.bfloat16)
            xl = torch.zeros_like(x) if split else None
            y = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
            st = torch.cuda.current_stream()

            def call():
                m.prefill_gemm(x.data_ptr(), xl.data_ptr() if split else None, M, y.data_ptr(), N, 2, st.cuda_stream)

            call()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(iters):
                call()
            e1.record(st)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / iters
            tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            pt = {"M": M, "K": K, "N": N, "ms": round(ms, 4), "tflops": round(tf, 1),
                  "frac": round(tf / peak_tflops, 4)}
            if M <= 64:  # the small-M kernel (exact codes in tensor memory): weight-stream bound
                pt["kernel"] = "decode_gemm_kernel"
                pt["weights_gb_s"] = round(N * K * 0.53125 / (ms * 1e-3) / 1e9, 1)
            out.append(pt)
            del x, xl, y
        m.close()
        torch.cuda.empty_cache()
    return {"workload": "config3: W4A16 g64 prefill GEMM sweep, bf16 activations, int4 -> bf16 in shared memory",
            "kernel": "prefill_gemm_kernel" + ("<split, 128>" if split else "<1 pass, 256>") + " (M > 64)",
            "mode": "split-bf16 (3 products)" if split else "one bf16 pass", "unit": "TFLOP/s",
            "peak_tflops": peak_tflops, "peak_kind": "measured bf16 (cuBLAS burst)", "points": out}


def tp_decode(pkg, model_dir, rank, world, local, ids, steps, warmup, kv_fp16, n_layers):
    """Tensor-parallel decode of ONE sequence over all `world` GPUs (xq_tp_*): every rank holds
    1/world of each matrix, two NCCL all-reduces of the hidden vector per layer and one 8-byte
    all-gather per token. Token-serial prefill of the same prompt on every rank, `warmup` steps
    (graph capture), then `steps` timed steps; the rate is steps / max-over-ranks device time.
    This is strong scaling of a single stream, reported beside the replica headline."""
    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")  # 16 KB all-reduces: plain peer transfers suffice
    uid = [pkg.Tp.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    t = pkg.Tp(model_dir, world, rank, uid[0], max_context=len(ids) + warmup + steps + 8, device=local,
               kv_fp16=kv_fp16)
    try:
        t.prefill(ids)
        t.decode(max(1, warmup))
        dist.barrier()
        ms, toks = t.decode(steps)
        ms_max = max_over_ranks(ms, world)
    finally:
        t.close()
    return {"tok_s": round(steps / (ms_max / 1000.0), 2), "ms_per_token": round(ms_max / steps, 4),
            "n_gpus": world, "steps": steps, "prompt": len(ids),
            "collectives_per_token": {"all_reduce_hidden_f32": 2 * n_layers, "all_gather_8_bytes": 1},
            "api": "xq_tp_decode (CUDA graph per step with the NCCL calls captured)",
            "scaling": "strong (one sequence; 1/world of the weights per GPU)",
            "tokens_head": [int(v) for v in toks[:8]]}


def config4_batched(pkg, model_dir, peak_gbs, weight_bytes, batches=(1, 8, 64), steps=64, prompt=PROMPT_LEN,
                    kv_fp16=False):
    """Config 4: batched decode of the 9B package, B independent sequences with their own
    512-token random prompts (xq_batch_*: one weight pass per step for all B tokens). value =
    B * steps / CUDA-event time of `steps` graph-launched steps (after the untimed capture step).
    Algorithmic bytes per step: every weight once (codes + fp16 scales), plus per sequence its
    DeltaNet recurrent and conv states read and written and its KV cache read at the mean timed
    context and one row written."""
    out = []
    kv_elem = 2 if kv_fp16 else 4
    for B in batches:
        b = pkg.Batch(model_dir, batch=B, max_context=prompt + steps + 8, kv_fp16=kv_fp16)
        rng = np.random.default_rng(SEED + 4000 + B)
        for i in range(B):
            b.prefill(i, rng.integers(0, 248320, prompt).astype(np.int32))
        ms, toks = b.decode_timed(steps)
        b.close()
        ctx = prompt + 1 + steps / 2
        per_seq = 24 * (2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4) + 8 * 2 * 4 * 256 * kv_elem * (ctx + 1)
        alg = weight_bytes + B * per_seq
        us = ms / steps * 1000
        out.append({"batch": B, "tok_s": round(B * steps / (ms / 1000.0), 1), "us_per_step": round(us, 1),
                    "algorithmic_bytes_per_step": int(alg),
                    "roofline": {"bound": "hbm", "achieved": round(alg / (us * 1e-6) / 1e9, 1), "peak": peak_gbs,
                                 "unit": "GB/s", "frac": round(alg / (us * 1e-6) / 1e9 / peak_gbs, 4)},
                    "tokens_head": [int(v) for v in toks[0, :4]]})
    return {"workload": "config4: batched decode of the 9B-shaped package, B sequences with independent 512-token "
                        "random prompts, greedy", "steps_timed": steps, "kv_dtype": "f16" if kv_fp16 else "f32",
            "engine": "xq_batch_decode_timed: CUDA graph per step, tcgen05 split-bf16 GEMMs with M = B",
            "points": out}


def cpu_baseline(model_dir, steps, preset="cfg2", prompt=PROMPT_LEN, warmup=0):
    """The reference's own CPU path (compiled from its sources) on the same package and context,
    on a bounded sample: a `prompt`-token prefill and `warmup` decode tokens (untimed), then
    `steps` greedy decode tokens through its C ABI, timed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    cores = min(8, os.cpu_count() or 1)
    ids = np.random.default_rng(SEED).integers(0, 248320, prompt).astype(np.int32)
    if oracle.ref_available():
        s = oracle.RefSession(model_dir, threads=cores)
        kind = "reference"
    else:
        oracle.port().xo_set_threads(cores)
        s = oracle.PortModel(model_dir)
        kind = "port"
    s.prefill(ids)
    for _ in range(warmup):
        s.decode_one()
    t = time.time()
    for _ in range(steps):
        s.decode_one()
    dt = time.time() - t
    s.close()
    return dict({"value": round(steps / dt, 4), "unit": "tok/s", "cores": cores, "kind": kind,
                 "sample": f"{steps} greedy decode steps after a {prompt}-token prompt and {warmup} untimed "
                           f"steps (context {prompt + warmup}..{prompt + warmup + steps}) on the "
                           f"{'9B' if preset == 'cfg2' else preset} package; the "
                           f"reference's WorkerPool caps at min(8, hardware_concurrency) threads"}, **host_cpu())


def max_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    """The largest per-rank value of x (a rank's timed duration): every rank takes the same
    collective steps; with world == 1 it is x itself."""
    if world <= 1:
        return float(x)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(units_per_rank: int, world: int, seconds_max: float) -> float:
    """Whole-job throughput of replicas: all ranks' units over the slowest rank's time."""
    return world * units_per_rank / seconds_max


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    __graft_entry__.load_package()  # registers the package module for the synthetic data generator
    d = make_package(0, 1, args.preset)
    steps = max(1, min(args.steps, 16))
    warm = max(0, min(args.warmup, 3))  # untimed decode steps after the prompt (~1 s each on the host)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    prompt = min(args.prompt, PROMPT_LEN)
    cb = cpu_baseline(d, steps, args.preset, prompt=prompt, warmup=warm)
    line = {"metric": METRIC, "value": cb["value"], "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": round(1000.0 / cb["value"], 2) if cb["value"] else None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init package)",
            "config": {"workload": "config2: Qwen3.5-9B-shaped W4A16 g64, 32 layers, vocab 248320, greedy decode"
                       if args.preset == "cfg2" else f"{args.preset} preset (functional check, not a bench line)",
                       "prompt": prompt, "kv_dtype": "f32", "cpu_sample": True},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not oracle.ref_available():
        line["cpu_baseline"]["kind"] = "port"
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kv-fp16", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=12)
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN, help="prompt length (512 = the benchmark shape)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config-0 GEMV and config-1 step lines")
    ap.add_argument("--no-tp", action="store_true", help="N > 1: skip the tensor-parallel single-sequence line")
    ap.add_argument("--cpu-prompt", type=int, default=32,
                    help="prompt tokens before the cpu_baseline's timed decode steps (its prefill runs at the "
                         "reference's ~2.5 tok/s; the reference arm keeps --prompt)")
    ap.add_argument("--gemm-only", default=None, metavar="M,K,N",
                    help="time only the prefill GEMM at one config-3 shape (profiling runs), print its point")
    ap.add_argument("--gemm-split", action="store_true", help="with --gemm-only: the split-bf16 mode")
    ap.add_argument("--gemv-cost-only", action="store_true",
                    help="only the standalone GEMV's fixed-cost fit (gemv_fixed_cost)")
    ap.add_argument("--batch-only", type=int, default=0, metavar="B",
                    help="time only batched decode (config 4) at batch B, --steps steps (profiling runs)")
    ap.add_argument("--preset", default="cfg2", choices=["cfg2", "small"],
                    help="synthetic package: cfg2 = the benchmark's 9B shape; small = a quick functional check")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    if args.gemv_cost_only:
        pkg = __graft_entry__.load_package()
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(gemv_fixed_cost(pkg, peaks()[0])), flush=True)
        return 0
    if args.gemm_only:
        M, K, N = (int(v) for v in args.gemm_only.split(","))
        pkg = __graft_entry__.load_package()
        r = config3_sweep(pkg, bf16_peak(), iters=args.steps, split=args.gemm_split, shapes=((K, N),), m_values=(M,))
        print(json.dumps(r), flush=True)
        return 0
    if args.batch_only:
        pkg = __graft_entry__.load_package()
        d = make_package(0, 1, args.preset)
        import torch

        torch.cuda.set_device(0)
        w = json.loads(pkg.Session(d, device=0).json("backend")).get("weight_bytes", 0)
        peak, _ = peaks()
        r = config4_batched(pkg, d, peak, w, batches=(args.batch_only,), steps=args.steps, kv_fp16=args.kv_fp16)
        print(json.dumps(r), flush=True)
        return 0
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=900))
    pkg = __graft_entry__.load_package()
    d = make_package(rank, world, args.preset)
    if world > 1:
        dist.barrier()
    sess = pkg.Session(d, device=local, kv_fp16=args.kv_fp16, max_context_tokens=args.prompt + args.warmup +
                       args.steps + 128)
    ids = np.random.default_rng(SEED + rank).integers(0, 248320, args.prompt).astype(np.int32)
    m = sess.prefill(ids)
    prefill_tok_s = m.prefill_tokens_per_second
    h_serial = sess.hidden()
    sess.decode_timed(args.warmup)  # untimed warm-up steps (graph capture happens here)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        dev_ms, toks = sess.decode_timed(args.steps, want_tokens=True)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(dev_ms, world)
    value = job_rate(args.steps, world, ms_max / 1000.0)

    # e2e: the same metric through xq_decode_one (host API call; 4-byte token read back per step)
    e2e_steps = min(args.steps, 64)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        sess.decode_one()
    e2e_s = time.perf_counter() - t0
    e2e_value = job_rate(e2e_steps, world, max_over_ranks(e2e_s, world))

    # one sequence sharded over every GPU of the job (tensor parallel), all ranks together
    tp = None
    if world > 1 and not args.no_tp:
        tp_ids = np.random.default_rng(SEED).integers(0, 248320, args.prompt).astype(np.int32)
        try:  # a shape that does not split evenly fails the same way on every rank, before NCCL
            tp = tp_decode(pkg, d, rank, world, local, tp_ids, args.steps, args.warmup, args.kv_fp16,
                           32 if args.preset == "cfg2" else 2)
        except (RuntimeError, ValueError) as e:
            tp = {"error": str(e)[:300]}

    info = json.loads(sess.json("backend"))
    if os.environ.get("XQ_STEP_TRACE") and rank == 0 and info.get("step_phase_trace"):
        # per-phase device timestamps of the step kernel (slower steps: every step syncs)
        print(json.dumps({"step_phase_trace": info["step_phase_trace"]}), file=sys.stderr, flush=True)
    kernels_per_step = int(info.get("kernels_per_decode_step", 0))
    peak, peak_kind = peaks()
    # standalone GEMVs of the kernel ABI: both engines at the gate+up and the lm_head shapes
    gemvs = [gemv_roofline(pkg, peak, engine=e, rows=r) for r in (24576, 248320) for e in ("dp4a", "mma")] \
        if rank == 0 else None
    gemv = gemvs[0] if gemvs else None
    # batched prefill through the tensor-core GEMMs: a second session on the shared weights
    sb = pkg.Session(d, device=local, kv_fp16=args.kv_fp16, max_context_tokens=args.prompt + 64, prefill_batched=True)
    sb.prefill(ids)  # first call allocates its buffers
    mb = sb.prefill(ids)
    prefill_batched = {"value": round(mb.prefill_tokens_per_second, 1), "unit": "tok/s",
                       "prompt": args.prompt, "hidden_rel_err_vs_token_serial":
                       float(np.abs(sb.hidden() - h_serial).max() / max(1e-30, np.abs(h_serial).max())),
                       "path": "tcgen05 GEMMs (split-bf16) + sequence kernels; xq_prefill wall time"}
    sb.close()
    # the per-config lines run at N = 1 (at N > 1 the job measures replicas and tensor parallel)
    extra = world == 1 and not args.no_extra
    cfg0 = config0_gemv(pkg, peak) if extra else None
    gemv_cost = gemv_fixed_cost(pkg, peak) if extra else None
    cfg3 = config3_sweep(pkg, bf16_peak()) if extra else None
    cfg4 = config4_batched(pkg, d, peak, info.get("weight_bytes", 0), kv_fp16=args.kv_fp16) \
        if extra and args.preset == "cfg2" else None
    cfg1 = config1_step(pkg, peak, args.kv_fp16) if extra else None
    step_bytes = info.get("weight_bytes", 0)
    if rank == 0:
        # Algorithmic bytes of one decode step: every weight matrix once (codes + fp16 scales),
        # the DeltaNet recurrent and conv states read and written, the KV cache read (mean
        # context over the timed steps) and written, the embedding row.
        ctx0 = args.prompt + args.warmup
        kv_elem = 2 if args.kv_fp16 else 4
        kv_bytes = 8 * 2 * 4 * 256 * kv_elem * (ctx0 + args.steps / 2 + 1)
        state_bytes = 24 * (2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4)
        alg_step = step_bytes + state_bytes + kv_bytes + 4096 * 2
        ms_step = ms_max / args.steps
        roof = step_roofline(alg_step, ms_step, peak)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init 9B-shaped package)",
            "config": {"workload": "config2: Qwen3.5-9B-shaped W4A16 g64 (32 layers, 3:1 DeltaNet:GQA, vocab "
                                   "248320), 512-token random prompt, greedy decode, batch 1",
                       "prompt": args.prompt, "context_during_timing": [args.prompt + args.warmup,
                                                                         args.prompt + args.warmup + args.steps],
                       "kv_dtype": "f16" if args.kv_fp16 else "f32", "parallelism": f"replicas{world}",
                       "l2": "inputs larger than L2 (4.3 GB of weights streamed per step)",
                       "step_execution": "persistent cooperative kernel" if info.get("persistent_step_kernel")
                       else "CUDA graph of per-op kernels with PDL",
                       "step_gemv": "integer tensor cores (mma.sync m16n8k32 u8 x s8, exact s32)"
                       if info.get("tensor_core_gemv") else "dp4a"},
            "prefill_tok_s": round(prefill_tok_s, 2),
            "roofline": dict(roof, peak_kind=peak_kind),
            "gemv_kernel": dict(gemv, peak_kind=peak_kind) if gemv else None,
            "gemv_kernels": [dict(g, peak_kind=peak_kind) for g in gemvs] if gemvs else None,
            "prefill_batched_tok_s": prefill_batched,
            "config0_gemv": cfg0,
            "gemv_fixed_cost": gemv_cost,
            "config3_gemm": cfg3,
            "config4_batched_decode": cfg4,
            "config1_step": cfg1,
            "tensor_parallel_decode": tp,
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
                    "api": "xq_decode_one"},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clk.summary(),
            "tokens_head": [int(v) for v in toks[:8]],
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(d, args.cpu_steps, args.preset, prompt=args.cpu_prompt)
        if args.preset != "cfg2":
            line["config"]["workload"] = f"{args.preset} preset (functional check, not a bench line)"
        print(json.dumps(line), flush=True)
    sess.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
