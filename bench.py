"""Benchmark: SAM ViT-H image encoder with SparseSAM (density 0.3) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: launched by torchrun, one rank per GPU)
    python bench.py --mode attn | mlp   (BASELINE configs 1 / 2, one GPU, one JSON line per case)
    python bench.py --mode predictor    (the SAM-HQ evaluation step: encoder + box-prompted HQ decode)

A step is one SparseSAM-patched encoder forward over one batch of synthetic
1024x1024 images (batch 64 per GPU; images are independent shards, no collective
on the data path -> weak scaling). Prints ONE JSON line on rank 0:

  value  images/s over all ranks with the batch already in HBM (device-timed,
         CUDA events, barrier + synchronize on both sides, max over ranks)
  e2e    the same metric through the public API with host buffers: pinned host
         images -> device, encoder(x), features -> host, every step's copies inside
         the timed region; serving-style double buffering (uploads and downloads on
         a copy stream, overlapped with the neighbouring steps' forwards)
  roofline  the dominant kernel (the tcgen05 GEMM): algorithmic TFLOP/s from CUDA
         events around its launches in a separate pass after the timed region
         (the timed region itself carries no per-launch events) vs the measured peak
  cpu_baseline  the CPU restatement of the reference path (oracle/) on the host
         cores, rank 0 at N=1, on a bounded sample (one image)

--impl reference times the reference's CPU path (the oracle restatement: the
reference's own GPU kernel is a CuTe-DSL SM80 JIT that is not part of this
build) with all host threads, on the same metric, one image per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "SAM ViT-H encoder images/sec @1024², d=0.3, bf16, 1/2/4/8 B200; % TC peak"
ARCH = "vit_h"
PER_GPU_BATCH = 64
RATIO = 0.3
IMG = 1024


def encoder_stream_gb(arch: str, batch: int, img: int = 1024) -> tuple:
    """(bf16 weights of the blocks, one block's activations) in GB for `batch` images:
    12 C^2 weights per block; the fp32 residual rows plus the bf16 qkv rows of the
    padded 14x14 window grid."""
    from sparsesam_b200.host import VIT_CONFIGS
    cfg = VIT_CONFIGS[arch]
    C, depth = cfg["embed_dim"], cfg["depth"]
    T = (img // 16) ** 2
    Tp = (-(-(img // 16) // 14) * 14) ** 2
    return depth * 12 * C * C * 2 / 1e9, batch * (T * C * 4 + Tp * 3 * C * 2) / 1e9


def encoder_flops(arch: str, ratio: float, img: int = 1024, mlp_merge: bool = True) -> float:
    """Algorithmic FLOPs per image, valid-token convention: qkv/proj on the real
    tokens, windowed attention over valid queries x enabled keys, global attention
    over enabled 64x64 block pairs, MLP at keep_n in the sparse-MLP blocks, plus
    patch embedding and neck; LN / softmax / rel-pos / scoring excluded."""
    from oracle.order import a_shape_n_init, keep_n_for
    from sparsesam_b200.host import VIT_CONFIGS
    cfg = VIT_CONFIGS[arch]
    C, depth, heads, gidx = cfg["embed_dim"], cfg["depth"], cfg["num_heads"], set(cfg["global_attn_indexes"])
    d = C // heads
    g = img // 16
    T = g * g
    fl = 2.0 * T * 768 * C                                     # patch embedding
    seen_global = False
    for i in range(depth):
        fl += 2.0 * T * C * 4 * C                              # qkv + proj
        if i in gidx:
            nb = -(-T // 64)
            n_init = a_shape_n_init(T, 64, ratio, True)
            pairs = sum(64 * (min(n_init, nb) * 64 + (64 if m >= n_init else 0)) for m in range(nb))
            fl += 4.0 * d * heads * pairs
        else:
            keys = min(a_shape_n_init(196, 64, ratio, False) * 64, 196)
            fl += 4.0 * d * heads * T * keys
        sparse_mlp = mlp_merge and ratio < 1.0 and i not in gidx and seen_global
        rows = keep_n_for(ratio, T) if sparse_mlp else T
        fl += 2.0 * 2 * rows * C * 4 * C                       # fc1 + fc2
        seen_global = seen_global or i in gidx
    fl += 2.0 * T * (C * 256 + 9 * 256 * 256)                  # neck
    return fl


def _peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": p["bf16_tflops"], "bf16_tflops_sustained": p["bf16_tflops_sustained"],
                "hbm_gbs": p["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(sample_images: int = 1) -> dict:
    """The CPU restatement (oracle/) of the reference path on this host's cores."""
    import torch

    from oracle import encoder as oenc
    from sparsesam_b200 import host
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    enc = host.build_image_encoder(ARCH, seed=0).eval()
    img = host.synthetic_images(sample_images, seed=0, img_size=IMG)
    t0 = time.perf_counter()
    oenc.encoder_forward(enc, img, RATIO)
    dt = time.perf_counter() - t0
    return {"value": sample_images / dt, "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"{sample_images} image(s) of the same workload (ViT-H, 1024^2, d={RATIO}), fp32 torch on CPU,"
                      f" {dt:.1f} s"}


def cpu_baseline_predictor(arch: str, ratio: float) -> dict:
    """The predictor step's CPU restatement (oracle/: the patched encoder and the
    box-prompted HQ decode with its mask resize) on this host's cores, one image."""
    import torch

    from oracle import decoder as odec
    from oracle import encoder as oenc
    from sparsesam_b200 import hq
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    sam = hq.build_sam_hq(arch)
    sd = sam.state_dict()
    images, _, boxes = hq.synthetic_box_batch(1, seed=0, img_size=IMG)
    t0 = time.perf_counter()
    with torch.no_grad():
        feats, interm = oenc.encoder_forward(sam.image_encoder, sam.preprocess(images), ratio)
        low, _ = odec.decode_boxes(sd, feats, interm[0], boxes, (IMG, IMG), False, True)
        _ = odec.postprocess(low, IMG, (IMG, IMG), (IMG, IMG)) > 0
    dt = time.perf_counter() - t0
    return {"value": 1 / dt, "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"1 image of the same workload ({arch}, 1024^2, d={ratio}: encoder fp32, decode fp64), "
                      f"torch on CPU, {dt:.1f} s"}


def shard_seed(rank: int) -> int:
    """Seed of rank `rank`'s image shard: every rank encodes its own images."""
    return 1000 + rank


def max_over_ranks(ms: float, world: int, device) -> float:
    """The slowest rank's time (the job ends when its last rank does); `world` 1: ms."""
    if world <= 1:
        return ms
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(per_rank_batch: int, world: int, steps: int, ms: float) -> float:
    """Images/s of the whole job: every rank's images over the slowest rank's time."""
    return per_rank_batch * world * steps / (ms * 1e-3)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from oracle import encoder as oenc
    from sparsesam_b200 import host
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    enc = host.build_image_encoder(ARCH, seed=0).eval()
    img = host.synthetic_images(1, seed=0, img_size=IMG)
    for _ in range(min(args.warmup, 1)):
        oenc.encoder_forward(enc, img, RATIO)
    steps = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for _ in range(steps):
        oenc.encoder_forward(enc, img, RATIO)
    dt = (time.perf_counter() - t0) / steps
    v = 1.0 / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "images/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"SAM ViT-H encoder 1024x1024, d={RATIO}, one image per step (CPU sample)",
                       "global_batch": 1, "ratio": RATIO},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": "one ViT-H image per step through the oracle restatement of the reference "
                                       "path (the reference's own kernel is a CuTe-DSL SM80 JIT)"},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from sparsesam_b200 import _lib, host, ops, registry

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # NCCL's own log lines (with NCCL_DEBUG set) go to stderr: stdout carries the one JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    batch = args.batch
    arch, ratio = args.arch, args.ratio
    enc = host.build_image_encoder(arch, seed=0, device=dev).eval()
    if ratio < 1.0:
        registry.apply_sam(enc, "sparsesam", ratio=ratio)
    else:  # the dense control: apply_sam treats ratio >= 1 as no patch (registry.py:65-66)
        from sparsesam_b200.sparsesam.sam import apply_patch
        apply_patch(enc, ratio=1.0)
    # each rank owns its own shard of images (seeded by rank)
    x_host = host.synthetic_images(batch, seed=shard_seed(rank), img_size=IMG).pin_memory()
    x_dev = x_host.to(dev)
    feat_host = torch.empty(batch, 256, IMG // 16, IMG // 16, dtype=torch.float32).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(fn, steps):
        barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(s.elapsed_time(e), world, dev)

    with torch.no_grad():
        def step_device():
            enc(x_dev)

        copy_stream = torch.cuda.Stream(dev)
        main = torch.cuda.current_stream(dev)
        x_buf = [torch.empty_like(x_dev) for _ in range(2)]
        feat_buf = [feat_host, torch.empty_like(feat_host).pin_memory()]

        def run_e2e(steps):
            # step i+1's images upload on the copy stream while step i computes, and
            # step i's features download there while step i+1 computes
            start = torch.cuda.Event()
            start.record(main)
            in_ready = [torch.cuda.Event(), torch.cuda.Event()]
            consumed = [torch.cuda.Event(), torch.cuda.Event()]

            def upload(i):
                b = i % 2
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_event(start if i < 2 else consumed[b])  # buffer b free again
                    x_buf[b].copy_(x_host, non_blocking=True)
                    in_ready[b].record(copy_stream)

            upload(0)
            for i in range(steps):
                b = i % 2
                if i + 1 < steps:
                    upload(i + 1)
                main.wait_event(in_ready[b])
                feats, _ = enc(x_buf[b])
                consumed[b].record(main)
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_event(consumed[b])
                    feats.record_stream(copy_stream)
                    feat_buf[b].copy_(feats, non_blocking=True)
            main.wait_stream(copy_stream)

        for _ in range(args.warmup):
            step_device()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        launches0 = _lib.launch_count
        ms = timed(step_device, args.steps)
        launches = (_lib.launch_count - launches0) // max(1, args.steps)
        clk = clocks.stop()
        # per-kernel pass (its own steps, outside the timed region): CUDA events
        # around every GEMM / attention launch on the launching stream
        kernel_steps = max(1, min(args.steps, 3))
        ops.KernelTimer.records = []
        ops.KernelTimer.active = True
        timed(step_device, kernel_steps)
        ops.KernelTimer.active = False
        run_e2e(2)
        ms_e2e = timed(lambda: run_e2e(args.steps), 1)
        # the pipelined copies deliver the same features as a plain forward
        ref = enc(x_dev)[0].cpu()
        torch.cuda.synchronize()
        e2e_err = (feat_buf[(args.steps - 1) % 2] - ref).abs().max().item()
        if not e2e_err <= 2e-2:
            raise RuntimeError(f"end-to-end features differ from the device forward (max abs {e2e_err})")
    err = ops.device_error()
    if err != 0:
        raise RuntimeError(f"device error flag {err}")

    # dominant kernel: the GEMM (tcgen05); per-launch averages over the timed region
    g = [(fl, st.elapsed_time(en)) for kind, fl, st, en in ops.KernelTimer.records if kind == "gemm"]
    a = [(fl, st.elapsed_time(en)) for kind, fl, st, en in ops.KernelTimer.records if kind.startswith("attention")]
    a_win = sum(st.elapsed_time(en) for kind, _, st, en in ops.KernelTimer.records if kind == "attention_window")
    a_glb = sum(st.elapsed_time(en) for kind, _, st, en in ops.KernelTimer.records if kind == "attention_global")
    peaks = _peaks()
    g_tflops = sum(f for f, _ in g) / (sum(t for _, t in g) * 1e-3) / 1e12 if g else None
    a_tflops = sum(f for f, _ in a) / (sum(t for _, t in a) * 1e-3) / 1e12 if a else None
    gemm_ms_step = sum(t for _, t in g) / kernel_steps
    attn_ms_step = sum(t for _, t in a) / kernel_steps

    value = job_throughput(batch, world, args.steps, ms)
    e2e = job_throughput(batch, world, args.steps, ms_e2e)
    flops_img = encoder_flops(arch, ratio)
    enc_tflops = flops_img * value / world / 1e12          # per GPU
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    traffic = None
    tpath = os.path.join(REPO, "profiles", "gemm_traffic.json")
    if arch == "vit_h" and os.path.exists(tpath):
        # captured on ViT-H at batch 8; GEMM rows (tokens) and with them the bytes grow with the batch
        with open(tpath) as f:
            t = json.load(f)
        traffic = t["bytes_per_launch_at_batch8"] * batch / t["measured_at_batch"]
    img_mb = x_host.numel() * 4 / 1e6
    line = {
        "metric": METRIC if (arch, ratio) == (ARCH, RATIO) else
        f"SAM {arch} encoder images/sec @1024², d={ratio}, bf16, B200; % TC peak",
        "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"SAM {arch} image encoder ({dict(vit_h='configs[4]', vit_l='configs[3]', vit_b='configs[0]')[arch]}), "
                               f"1024x1024, SparseSAM density {ratio}, "
                               f"{batch} images per GPU, seed-0 random weights",
                   "global_batch": batch * world, "per_gpu_batch": batch, "ratio": ratio,
                   "parallelism": f"dp{world} (independent image shards, no collective)",
                   "l2": "inputs larger than L2 (126 MB): each step streams {:.0f} MB of images, {:.2f} GB of "
                         "bf16 weights and {:.2f} GB of block activations".format(img_mb, *encoder_stream_gb(arch, batch))},
        "e2e": {"value": e2e, "unit": "images/s", "h2d_bytes_per_step": x_host.numel() * 4,
                "d2h_bytes_per_step": feat_host.numel() * 4},
        "gpu_launches": launches,
        "tc_peak_frac": {"encoder_tflops_per_gpu": enc_tflops, "flops_per_image": flops_img,
                         "peak_tflops": peaks["bf16_tflops"], "frac": enc_tflops / peaks["bf16_tflops"],
                         "peak_source": peaks["source"] + " burst bf16"},
        "roofline": {"kernel": "gemm_bf16_tn (tcgen05)", "bound": "tensor", "achieved": g_tflops,
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": (g_tflops / peaks["bf16_tflops_sustained"]) if g_tflops else None,
                     "traffic": traffic, "peak_source": peaks["source"] + " sustained bf16",
                     "gemm_ms_per_step": gemm_ms_step, "attention_ms_per_step": attn_ms_step,
                     "attention_window_ms_per_step": a_win / kernel_steps,
                     "attention_global_ms_per_step": a_glb / kernel_steps,
                     "attention_tflops": a_tflops,
                     "achieved_from": "algorithmic FLOPs (2*M*N*K per GEMM; the fp32-accurate split GEMMs of the "
                                      "stem and neck counted at their unsplit K) over CUDA-event durations from a "
                                      f"separate {kernel_steps}-step pass"},
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(1)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _event_ms(fn, steps: int) -> float:
    """Mean CUDA-event time of fn() over `steps` calls on the current stream."""
    import torch
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def _micro_common(args, dev):
    from sparsesam_b200 import ops
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--mode attn / mlp / predictor are single-GPU benchmarks")
    return ops, _peaks()


def run_attn_micro(args) -> None:
    """Stripe-Sort block-sparse attention at SAM global-attention
    shapes (B=8, heads=16, N=4096 from a 64x64 grid, d=64, bf16; Q/K/V ~ N(0,1)
    seed 1, rel-pos tables (127, 64) ~ N(0, 0.02)); the permutation is Stripe-Sort
    of the same K (sam.py:193-209); densities 0.3 / 0.4 / 0.5 and the dense
    control, on the reference's 64-token mask blocks and on 128-token blocks.
    One JSON line per (mask block, density) plus one for the Stripe-Sort kernel."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops, peaks = _micro_common(args, dev)
    B, heads, win, d = 8, 16, 64, 64
    N, C = win * win, heads * d
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(B * N, 3 * C, generator=g).to(torch.bfloat16).to(dev)
    th = (torch.randn(2 * win - 1, d, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    tw = (torch.randn(2 * win - 1, d, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    base = ops.zorder(win, win, dev)[0]
    k_view = qkv[:, C:]

    def sort():
        return ops.stripe_sort_perm(k_view, B, heads, win, win, d, base, ld=qkv.stride(0))
    perm = sort()[0]
    for _ in range(args.warmup):
        sort()
    ms_sort = _event_ms(sort, args.steps)
    # algorithmic bytes: K read twice (two passes over the groups), three int32 rows written
    sort_bytes = B * heads * (2 * N * d * 2 + 3 * N * 4)
    common = {"data": "synthetic", "dtype": "bf16", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
              "l2": "qkv 201 MB and the bias workspace 134 MB exceed L2"}
    print(json.dumps({"metric": "Stripe-Sort permutation (BASELINE config 1 K)", "value": sort_bytes / ms_sort / 1e6,
                      "unit": "GB/s", "ms_per_call": ms_sort, "higher_is_better": True,
                      "roofline": {"bound": "hbm", "achieved": sort_bytes / ms_sort / 1e6, "peak": peaks["hbm_gbs"],
                                   "unit": "GB/s", "frac": sort_bytes / ms_sort / 1e6 / peaks["hbm_gbs"],
                                   "algorithmic_bytes": sort_bytes},
                      "config": {"workload": "stripe_sort_kernel, B*heads=128 rows of 4096 tokens, d=64"},
                      **common}), flush=True)
    for n_block in (64, 128):
        for ratio in (0.3, 0.4, 0.5, 1.0):
            n_init = ops.a_shape_n_init(N, n_block, ratio, True)
            out = torch.empty(B * N, C, dtype=torch.bfloat16, device=dev)

            def call():
                ops.sparse_attn(qkv, B, heads, win, d, th, tw, perm, n_init, True, d ** -0.5, out=out,
                                n_block=n_block)
            for _ in range(args.warmup):
                call()
            ms = _event_ms(call, args.steps)
            if ops.device_error() != 0:
                raise RuntimeError("device error flag raised")
            fl = ops.attention_flops(B * heads, N, d, n_init, True, n_block)
            tf = fl / ms / 1e9
            print(json.dumps({
                "metric": "Stripe-Sort attention TFLOP/s (BASELINE config 1)", "value": tf, "unit": "TFLOP/s",
                "ms_per_call": ms, "higher_is_better": True,
                "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tf / peaks["bf16_tflops"], "peak_source": peaks["source"] + " burst bf16",
                             "frac_of_sustained": tf / peaks["bf16_tflops_sustained"], "algorithmic_flops": fl},
                "config": {"workload": "B=8 x 16 heads, N=4096 (64x64), d=64, global A-shape mask with diagonal",
                           "density": ratio, "mask_block": n_block, "n_init_blocks": n_init,
                           "includes": "rel-pos bias pre-pass + attention (one ssam_sparse_attn_fwd call)"},
                **common}), flush=True)


def run_mlp_micro(args) -> None:
    """the Residual-Consistency MLP at ViT-L width. Tokens X
    [8, 4096, 1024] ~ N(0,1) seed 2 (bf16 values, held in the fp32 residual stream
    the MLP updates in place), LN weight 1 / bias 0, fc1 / fc2 trunc-normal 0.02
    with zero biases; the keep set is the reference's own rule (sam.py:273-280):
    Stripe-Sort group ranks of the tokens per head (X viewed as ViT-L's 16 heads of
    64 channels), summed over heads, the keep_n = round(r N) smallest, ties to the
    lowest index. One JSON line per keep fraction (0.3, 0.4)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops, peaks = _micro_common(args, dev)
    B, N, C, heads = 8, 4096, 1024, 16
    Hd = 4 * C
    g = torch.Generator().manual_seed(2)
    xb = torch.randn(B * N, C, generator=g).to(torch.bfloat16)
    x0 = xb.float().to(dev)
    xbf = xb.to(dev)
    from sparsesam_b200.host import _trunc_normal_
    w1, w2 = torch.empty(Hd, C), torch.empty(C, Hd)
    _trunc_normal_(w1, 0.02, g)
    _trunc_normal_(w2, 0.02, g)
    w1, w2 = w1.to(torch.bfloat16).to(dev), w2.to(torch.bfloat16).to(dev)
    b1 = torch.zeros(Hd, device=dev)
    b2 = torch.zeros(C, device=dev)
    lw = torch.ones(C, device=dev)
    lb = torch.zeros(C, device=dev)
    base = ops.zorder(64, 64, dev)[0]
    common = {"data": "synthetic", "dtype": "bf16", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
              "l2": "X is 134 MB in fp32 (> L2)"}
    for ratio in (0.3, 0.4):
        keep_n = max(1, round(ratio * N))

        def score():
            _, _, ipg = ops.stripe_sort_perm(xbf, B, heads, 64, 64, C // heads, base, ld=C)
            return ops.keep_select(ipg, B, heads, keep_n)
        rows = score()[1]
        x = x0.clone()
        ws = torch.empty(ops.rc_mlp_workspace_size(B * keep_n, C, Hd), dtype=torch.uint8, device=dev)

        def mlp():
            ops.rc_mlp(x, rows, B * keep_n, lw, lb, 1e-6, w1, b1, w2, b2, workspace=ws)
        xk = torch.empty(B * keep_n, C, dtype=torch.bfloat16, device=dev)
        h = torch.empty(B * keep_n, Hd, dtype=torch.bfloat16, device=dev)
        legs = {
            "score (Stripe-Sort + keep set)": score,
            "LN2 keep-row gather": lambda: ops.layernorm_gather(x, lw, lb, 1e-6, src_rows=rows, out=xk),
            "fc1 + GELU": lambda: ops.gemm_bf16(xk, w1, b1, epilogue=ops.SSAM_EPI_GELU_BF16, out=h),
            "fc2 + scatter-add": lambda: ops.gemm_bf16(h, w2, b2, epilogue=ops.SSAM_EPI_ADD_F32, out=x,
                                                       out_rows=rows),
        }
        for _ in range(args.warmup):
            mlp()
            for fn in legs.values():
                fn()
        ms = _event_ms(mlp, args.steps)
        leg_ms = {k: _event_ms(fn, args.steps) for k, fn in legs.items()}
        if ops.device_error() != 0:
            raise RuntimeError("device error flag raised")
        rk = B * keep_n
        fl = 2.0 * 2 * rk * C * Hd
        tf = fl / ms / 1e9
        ln_bytes = rk * C * (4 + 2)
        print(json.dumps({
            "metric": "RC-MLP TFLOP/s (BASELINE config 2)", "value": tf, "unit": "TFLOP/s", "ms_per_call": ms,
            "higher_is_better": True,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "peak_source": peaks["source"] + " burst bf16",
                         "frac_of_sustained": tf / peaks["bf16_tflops_sustained"], "algorithmic_flops": fl},
            "legs_ms": leg_ms,
            "ln_gather": {"bytes": ln_bytes, "gbs": ln_bytes / leg_ms["LN2 keep-row gather"] / 1e6,
                          "frac_of_hbm": ln_bytes / leg_ms["LN2 keep-row gather"] / 1e6 / peaks["hbm_gbs"]},
            "fc_tflops": {"fc1": fl / 2 / leg_ms["fc1 + GELU"] / 1e9, "fc2": fl / 2 / leg_ms["fc2 + scatter-add"] / 1e9},
            "config": {"workload": "RC-MLP on X [8, 4096, 1024], 1024->4096->1024 GELU, keep set of sam.py:273-280",
                       "keep_fraction": ratio, "keep_n": keep_n,
                       "timed": "ssam_rc_mlp_fwd (LN2 gather, fc1+GELU, fc2 scatter-add); scoring timed as a leg"},
            **common}), flush=True)


def run_predictor(args) -> None:
    """The HQ-44K evaluation step around the encoder (tasks/sam_hq44k/eval_hq44k.py:87-129)
    as a throughput benchmark: a step is preprocess -> patched encoder -> one
    box-prompted HQ decode per image (hq_token_only, the whole batch in one decoder
    pass) -> masks at 1024^2. Synthetic images with one ellipse each (the dataset is
    not available) and seeded random weights; the IoU printed is a pipeline check,
    not a quality figure. The timed step is captured once as a CUDA graph and
    replayed (hq.GraphedBoxStep): at small batches the eager step is launch-bound.
    value: images in HBM, device-timed; e2e: uint8 images from pinned host memory
    in and boolean masks out inside every step."""
    import torch
    from sparsesam_b200 import _lib, hq, registry
    from sparsesam_b200.sparsesam.sam import apply_patch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops, peaks = _micro_common(args, dev)
    arch, batch, ratio = args.arch, args.batch, args.ratio
    dec_dt = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[args.decoder_dtype]
    sam = hq.build_sam_hq(arch, device=dev, decoder_dtype=dec_dt)
    if ratio < 1.0:
        registry.apply_sam(sam.image_encoder, "sparsesam", ratio=ratio)
    else:
        apply_patch(sam.image_encoder, ratio=1.0)
    images, labels, boxes = hq.synthetic_box_batch(batch, seed=0, img_size=IMG)
    img_host = images.to(torch.uint8).pin_memory()
    box_host = boxes.pin_memory()
    img_dev, box_dev = img_host.to(dev), box_host.to(dev)
    mask_host = torch.empty(batch, 1, IMG, IMG, dtype=torch.bool).pin_memory()
    pred = hq.SamPredictor(sam)

    def encode(x_u8):
        x = sam.preprocess(x_u8)
        pred.features, pred.interm_features = sam.image_encoder(x)
        pred.original_size = pred.input_size = (IMG, IMG)
        pred.is_image_set = True

    def decode(bx):
        return pred.predict_torch(None, None, boxes=bx, hq_token_only=True)[0]

    def step():
        encode(img_dev)
        return decode(box_dev)

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        launches0 = _lib.launch_count
        eager_ms = _event_ms(step, args.steps)
        launches = (_lib.launch_count - launches0) // max(1, args.steps)
        enc_ms = _event_ms(lambda: encode(img_dev), args.steps)
        dec_ms = _event_ms(lambda: decode(box_dev), args.steps)
        # the timed step: the whole step captured once as a CUDA graph and replayed
        graphed = hq.GraphedBoxStep(sam, batch)

        def step_graph():
            return graphed(img_dev, box_dev)[0]

        def step_e2e():
            graphed.images.copy_(img_host, non_blocking=True)
            graphed.boxes.copy_(box_host, non_blocking=True)
            graphed.graph.replay()
            mask_host.copy_(graphed.masks, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        for _ in range(args.warmup):
            step_graph()
        torch.cuda.synchronize()
        clocks = ClockSampler(0)
        clocks.start()
        ms = _event_ms(step_graph, args.steps)
        clk = clocks.stop()
        step_e2e()
        ms_e2e = _event_ms(step_e2e, args.steps)
        masks = step_graph().clone()
        if not torch.equal(mask_host.to(dev), masks):
            raise RuntimeError("end-to-end masks differ from the device replay")
        iou = hq.compute_iou(masks, labels.to(dev)).item()
        biou = hq.compute_boundary_iou(masks[:4], labels[:4].to(dev)).item()
    if ops.device_error() != 0:
        raise RuntimeError("device error flag raised")
    flops_img = encoder_flops(arch, ratio)
    print(json.dumps({
        "metric": f"SAM-HQ predictor images/sec @1024², {arch}, d={ratio} (encoder + one box-prompted HQ decode "
                  "per image)",
        "value": batch / ms * 1e3, "unit": "images/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"bf16 encoder, {args.decoder_dtype} decoder", "data": "synthetic",
        "config": {"workload": f"SAM-HQ {arch} predictor: preprocess, SparseSAM encoder, HQ mask decoder with one "
                               "box per image in one decoder pass, masks upsampled to 1024x1024 "
                               "(eval_hq44k.py:87-129 step)",
                   "per_gpu_batch": batch, "ratio": ratio,
                   "l2": "inputs larger than L2: {:.0f} MB of images per step".format(img_host.numel() / 1e6)},
        "e2e": {"value": batch / ms_e2e * 1e3, "unit": "images/s", "h2d_bytes_per_step": img_host.numel() +
                box_host.numel() * 4, "d2h_bytes_per_step": mask_host.numel()},
        "legs_ms": {"encoder": enc_ms, "decode (prompt encoder, HQ decoder, mask upsampling)": dec_ms,
                    "eager step (no graph)": eager_ms},
        "timed": "the step captured once as a CUDA graph (hq.GraphedBoxStep) and replayed; legs and the eager "
                 "step from eager launches",
        "encoder_tflops": flops_img * batch / enc_ms / 1e9,
        "gpu_launches": launches,
        "iou_check": {"iou": iou, "boundary_iou_first4": biou,
                      "note": "random weights: a pipeline check, not segmentation quality"},
        "clocks": clk,
        **({} if args.no_cpu_baseline else {"cpu_baseline": cpu_baseline_predictor(arch, ratio)})}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=PER_GPU_BATCH)
    ap.add_argument("--ratio", type=float, default=RATIO, help="SparseSAM density (1.0: dense control)")
    ap.add_argument("--arch", choices=("vit_h", "vit_l", "vit_b"), default=ARCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decoder-dtype", choices=("fp16", "bf16", "fp32"), default="fp16",
                    help="predictor mode: the prompt encoder / HQ decoder dtype (the reference runs fp16)")
    ap.add_argument("--mode", choices=("encoder", "attn", "mlp", "predictor"), default="encoder",
                    help="encoder: the headline metric; attn / mlp: BASELINE configs 1 / 2 microbenchmarks; "
                         "predictor: the SAM-HQ evaluation step (encoder + box-prompted HQ decode)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "attn":
        run_attn_micro(args)
    elif args.mode == "mlp":
        run_mlp_micro(args)
    elif args.mode == "predictor":
        run_predictor(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
