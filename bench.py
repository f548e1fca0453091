"""Benchmark of the SpecCache Path-1 KV restore on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (default, one GPU): Llama-3-8B KV geometry — 32 layers x (K, V), 8 KV heads x
head_dim 128, T = 8192 tokens, per-(token, head) absmax INT8 codes with fp16 scales made
from fp16 N(0,1) values (seeded, synthetic), RoPE theta 5e5, one shift drawn uniformly
in [1, 4096] from the seed, bf16 output written into contiguous per-layer caches.

* ``value``: algorithmic HBM bytes of the fused restore (int8 K+V in, fp16 scales in,
  bf16 K+V out: 6*T*H*D + 4*T*H per layer) per second, inputs resident in HBM, one
  launch restoring all 32 layers per step.  1.62 GB per step exceeds the 126 MB L2, so
  no flush is needed between steps.
* ``e2e``: the same metric through the pinned-host restore pipeline
  (``sc_pipeline_restore``): every step copies the 32 layers' INT8 codes and scales
  from pinned host slabs (545 MB) and restores them, then reads back the last cache row
  of K and V.  ``restore_ms`` is the T=8192 restore time.
* ``cpu_baseline``: the reference's eager CPU arithmetic (the oracle port) on the host
  cores over a bounded sample (one layer).

With N > 1 (torchrun, one process per GPU) every rank restores its own 8-head shard of
an N x 8-head model (weak scaling, no collective on the data path); ``value`` is the
bytes of all ranks over the slowest rank's time.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

L_LAYERS, T_TOKENS, H_HEADS, D_HEAD = 32, 8192, 8, 128
THETA = 500000.0
CHUNK = 64
SEED = 0


def algorithmic_bytes(layers: int, tokens: int, heads: int, head_dim: int) -> int:
    """int8 K,V in + fp16 K,V scales in + bf16 K,V out."""
    return layers * (6 * tokens * heads * head_dim + 4 * tokens * heads)


def h2d_bytes(layers: int, tokens: int, heads: int, head_dim: int) -> int:
    return layers * (2 * tokens * heads * head_dim + 2 * 2 * tokens * heads)


def draw_shift(seed: int) -> int:
    return int(np.random.default_rng(seed).integers(1, 4097))


def read_peaks() -> tuple[float, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_profiled_traffic() -> float | None:
    """Per-launch DRAM bytes of the dense restore kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "dense_restore_llama8b_t8192_ncu.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch_full:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(",") for r in f if r.strip()]
        os.unlink(self.file.name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, smax, reasons, loaded = [], None, set(), []
        for r in rows:
            try:
                vals = [v.strip() for v in r]
                mhz, mx, util = float(vals[1]), float(vals[2]), float(vals[3])
            except (ValueError, IndexError):
                continue
            smax = mx
            sm.append(mhz)
            if util >= 50:
                loaded.append(mhz)
                for name, v in zip(names, vals[5:9]):
                    if v.lower() == "active":
                        reasons.add(name)
        pick = loaded or sm
        return {"sm_mhz": statistics.median(pick) if pick else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(loaded)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(scb, device, layers, tokens, heads, head_dim, seed):
    """Seeded fp16 N(0,1) K/V per layer, quantised on the GPU into [L, T, H, D] codes."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    kq = torch.empty((layers, tokens, heads, head_dim), dtype=torch.int8, device=device)
    vq = torch.empty_like(kq)
    ks = torch.empty((layers, tokens, heads, 1), dtype=torch.float16, device=device)
    vs = torch.empty_like(ks)
    for layer in range(layers):
        for q, s in ((kq, ks), (vq, vs)):
            x = torch.randn((tokens, heads, head_dim), generator=gen, device=device,
                            dtype=torch.float32).to(torch.float16)
            scb.quantize_kv_int8(x, q_out=q[layer], scale_out=s[layer])
    torch.cuda.synchronize(device)
    return kq, ks, vq, vs


def cpu_baseline_sample(layers_total: int, tokens: int, heads: int, head_dim: int, dp: int,
                        budget_s: float = 10.0) -> dict:
    """Time the oracle (the reference's eager CPU arithmetic) on one layer, host cores."""
    oracle = importlib.import_module("oracle.speccache_oracle")
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(SEED)
    kq = torch.randint(-127, 128, (tokens, heads, head_dim), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, (tokens, heads, head_dim), generator=g, dtype=torch.int8)
    ks = (torch.rand((tokens, heads, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)
    vs = (torch.rand((tokens, heads, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 5 or (time.perf_counter() < t_end and len(times) < 200):
        t0 = time.perf_counter()
        cos, sin = oracle.compute_rope_cos_sin_delta(dp, head_dim, THETA)
        oracle.dequant_rope_shift(kq, ks, cos, sin, out_dtype=torch.bfloat16)
        oracle.dequant_value(vq, vs, out_dtype=torch.bfloat16)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    per_layer = algorithmic_bytes(1, tokens, heads, head_dim)
    return {"value": per_layer / med / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 of {layers_total} layers (T={tokens}, H={heads}, D={head_dim}, K shift "
                      f"+ V dequant, bf16 out), median of {len(times)} runs; scales linearly per layer",
            "restore_ms_extrapolated": med * 1e3 * layers_total}


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    oracle = importlib.import_module("oracle.speccache_oracle")
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    dp = draw_shift(SEED)
    g = torch.Generator().manual_seed(SEED)
    t, h, d = T_TOKENS, H_HEADS, D_HEAD
    kq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    ks = (torch.rand((t, h, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)
    vs = (torch.rand((t, h, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)

    def step():
        cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, THETA)
        oracle.dequant_rope_shift(kq, ks, cos, sin, out_dtype=torch.bfloat16)
        oracle.dequant_value(vq, vs, out_dtype=torch.bfloat16)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    per_step = algorithmic_bytes(1, t, h, d)
    mean = sum(times) / len(times)
    value = per_step / mean / 1e9
    line = {
        "impl": "reference", "metric": "dequant+RoPE-shift GB/s (algorithmic bytes)",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 math, bf16 out",
        "data": "synthetic (seeded int8 codes, fp16 scales)",
        "config": {"workload": "llama3-8b KV restore sample: 1 layer of 32, T=8192, H=8, D=128, "
                               "theta=5e5, bf16 out", "layers_in_sample": 1, "seq_len": t,
                   "kv_heads": h, "head_dim": d, "delta_p": dp, "l2": "inputs > L2 n/a (CPU)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": "one layer of the 32-layer workload per step (reference eager "
                                   "arithmetic restated in torch-CPU, the oracle)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    scb = importlib.import_module("intelligent-bell_b200")
    from speccache_b200.cache import KVRestorePipeline

    layers, t, h, d = args.layers, T_TOKENS, H_HEADS, D_HEAD
    dp = draw_shift(SEED)
    kq, ks, vq, vs = make_inputs(scb, device, layers, t, h, d, SEED + 1000 * rank)
    k_out = torch.empty((layers, t, h, d), dtype=torch.bfloat16, device=device)
    v_out = torch.empty_like(k_out)
    per_step = algorithmic_bytes(layers, t, h, d)
    stream = torch.cuda.current_stream(device)

    def step():
        scb.restore_layers(kq, ks, vq, vs, delta_p=dp, theta=THETA, k_out=k_out, v_out=v_out)

    # ---- e2e set-up: pinned host slabs with the same codes ---------------------------
    n_blocks = t // CHUNK
    pipe = None if args.skip_e2e else KVRestorePipeline(layers, n_blocks, CHUNK, h, d, device=device,
                             max_restore_blocks=n_blocks, n_slots=3)
    if pipe is not None:
        pipe.k_quant.view(layers, t, h, d).copy_(kq.cpu())
        pipe.v_quant.view(layers, t, h, d).copy_(vq.cpu())
        pipe.k_scale.view(layers, t, h, 1).copy_(ks.cpu())
        pipe.v_scale.view(layers, t, h, 1).copy_(vs.cpu())
    e2e_k = [k_out[layer] for layer in range(layers)]
    e2e_v = [v_out[layer] for layer in range(layers)]
    block_ids = list(range(n_blocks))
    shifts = [dp] * n_blocks
    tail_host = torch.empty((2, h, d), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        pipe.restore(block_ids, shifts, e2e_k, e2e_v, theta=THETA)
        tail_host[0].copy_(k_out[layers - 1, t - 1], non_blocking=True)
        tail_host[1].copy_(v_out[layers - 1, t - 1], non_blocking=True)

    with ClockSampler(device.index if device.index is not None else 0) as clocks:
        # ---- value: kernel with inputs resident ------------------------------------------
        for _ in range(args.warmup):
            step()
        barrier(world)
        torch.cuda.synchronize(device)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        ev[0].record(stream)
        for i in range(args.steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
        launch_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
        total_ms = ev[0].elapsed_time(ev[-1])
        total_ms_max = max_over_ranks(total_ms, world, device)

        # ---- e2e: pinned host -> restore -> read back --------------------------------------
        e2e_ms = None
        if pipe is not None:
            for _ in range(args.warmup):
                e2e_step()
            torch.cuda.synchronize(device)
            barrier(world)
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            e1.record(stream)
            torch.cuda.synchronize(device)
            barrier(world)
            e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device)
    pipe_status = None
    if pipe is not None:
        pipe_status = pipe.status()
        pipe.close()

    if rank != 0:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    value = per_step * world * args.steps / (total_ms_max / 1e3) / 1e9
    avg_launch_ms = sum(launch_ms) / len(launch_ms)
    achieved = per_step / (avg_launch_ms / 1e3) / 1e9
    peak, peak_kind = read_peaks()
    traffic = read_profiled_traffic()
    e2e = None
    if e2e_ms is not None:
        e2e = {"value": per_step * world * args.steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
               "restore_ms": e2e_ms / args.steps,
               "h2d_bytes_per_step": h2d_bytes(layers, t, h, d),
               "d2h_bytes_per_step": int(tail_host.numel() * tail_host.element_size()),
               "h2d_gbs": h2d_bytes(layers, t, h, d) * world * args.steps / (e2e_ms / 1e3) / 1e9,
               "path": "sc_pipeline_restore from pinned host slabs, one kernel per layer",
               "gpu_launches": layers * args.steps, "device_status": pipe_status}
    line = {
        "metric": "dequant+RoPE-shift GB/s (algorithmic bytes) & % of B200 HBM peak; "
                  "T=8192 KV restore ms",
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 in, fp32 math, bf16 out",
        "data": "synthetic: seeded fp16 N(0,1) K/V quantised to int8 + fp16 scales",
        "config": {
            "workload": "llama3-8b KV restore: 32 layers x (K,V), T=8192, 8 KV heads x 128, "
                        "theta=5e5, one delta_p in [1,4096], bf16 contiguous per-layer caches",
            "layers": layers, "seq_len": t, "kv_heads_per_gpu": h, "head_dim": d,
            "delta_p": dp, "theta": THETA, "parallelism": f"kv-head shards x{world}",
            "l2": "inputs+outputs 1.62 GB per step > 126 MB L2 (no flush needed)",
        },
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.skip_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(layers, t, h, d, dp)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=L_LAYERS,
                    help="layers per step (32 = the workload; fewer only for profiling captures)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling aid: kernel leg only")
    ap.add_argument("--skip-cpu-baseline", action="store_true", help="profiling aid")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
