"""Benchmark of the SpecCache Path-1 KV restore on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama8b|paged|roundtrip|llama70b]

Workloads (synthetic, seeded data with the shapes and value distributions below):

* ``llama8b`` (default, the headline): Llama-3-8B KV geometry - 32 layers x (K, V),
  8 KV heads x head_dim 128, T = 8192 tokens, per-(token, head) absmax INT8 codes with
  fp16 scales made from fp16 N(0,1) values, RoPE theta 5e5, one shift drawn uniformly in
  [1, 4096] from the seed, bf16 output into contiguous per-layer caches.
  - ``value``: algorithmic HBM bytes of the fused restore per second (int8 K+V in, fp16
    scales in, bf16 K+V out: 6*T*H*D + 4*T*H per layer), inputs resident in HBM, one
    launch restoring all 32 layers per step.  Inputs + outputs are 1.62 GB per step, far
    above the 126 MB L2, so no flush is needed between steps.
  - ``e2e``: the same metric through the pinned-host restore pipeline
    (``sc_pipeline_restore``, the C ABI): each step copies the 32 layers' codes and
    scales from pinned host slabs (545 MB), restores them, and reads back the last cache
    row of K and V.  ``restore_ms`` is the T = 8192 restore time.  ``--block-order
    scattered`` restores the same 128 blocks from a slab of 256, every other block in a
    seeded random order (every block its own run: the fragmented pool of a long-running
    server) instead of consecutive ones.
  - ``e2e.h2d_ceiling_gbs``: the copy-only ceiling at the same N - every rank copies its
    whole pinned slab into HBM with nothing else running, all ranks at once, best of 5 -
    and ``e2e.h2d_vs_ceiling``, the pipeline's host-to-device rate over it;
    ``h2d_ceiling_sustained_gbs`` / ``h2d_vs_sustained_ceiling``: the same copy repeated
    back to back as many times as the timed restores.
  - ``cpu_baseline``: the reference's own eager functions (speccache/kernels/reference.py
    from the installed copy under baseline/_ref; the oracle port only if that import
    fails) on the host cores over a bounded sample (one layer).
  - N > 1 (torchrun): every rank restores its own 8-head shard of an N x 8-head model
    (weak scaling, no collective on the data path); ``value`` = bytes of all ranks over
    the slowest rank's time.  After the timing, ``gather_check``: every rank restores its
    heads of a small model into GPU 0's caches over NVLink (HeadShardGather), and GPU 0
    compares every bit with its own restore of all heads; a mismatch fails the run.
* ``paged``: ragged paged batch, Llama-3-8B geometry - 64 requests with lengths uniform
  in [256, 8192] and shifts uniform in [0, 4096] from the seed, INT8 pool of 64-token
  pages addressed by a shuffled page table, restored into packed bf16 caches in one
  launch.
* ``roundtrip``: Qwen-2.5-7B-like - 28 layers, 4 KV heads x 128, T = 16384, theta 1e6,
  fp16 N(0,1) K/V with 2% of channels scaled x10; quantize (bit-exact twin) then restore
  with shift 2048 into fp16.  ``offload``: every layer quantized on the GPU into the pinned
  slabs (``sc_pipeline_offload``); with ``--block-order scattered`` into every other block
  of a slab twice as large, in a seeded random order.
* ``llama70b``: Llama-3-70B KV geometry - 80 layers, 8 KV heads x 128, T = 32768, shift
  8192, theta 5e5; pinned host slab -> GPU pipeline; with N GPUs each rank restores 8/N
  heads (strong scaling).  ``value`` is end-to-end (H2D-bound).
* ``keyshift``: the RoPE shift of already-dequantised fp16 keys (the injector's
  apply_rope_shift), 32 layers x T = 8192 x 8 heads x 128, shift -384, one launch.

``--impl reference`` times the reference's own CPU implementation of the workload (as the
``cpu_baseline`` above) on all host threads; under torchrun rank 0 alone runs.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import json
import os
import random
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

SEED = 0
CHUNK = 64

WORKLOADS = {
    "llama8b": dict(layers=32, tokens=8192, heads=8, head_dim=128, theta=500000.0,
                    out=torch.bfloat16),
    "paged": dict(requests=64, min_len=256, max_len=8192, heads=8, head_dim=128, page=64,
                  theta=500000.0, out=torch.bfloat16),
    "roundtrip": dict(layers=28, tokens=16384, heads=4, head_dim=128, theta=1000000.0,
                      delta_p=2048, out=torch.float16),
    "llama70b": dict(layers=80, tokens=32768, heads=8, head_dim=128, theta=500000.0,
                     delta_p=8192, out=torch.bfloat16),
    "keyshift": dict(layers=32, tokens=8192, heads=8, head_dim=128, theta=500000.0,
                     delta_p=-384, out=torch.float16),
}


def restore_bytes(rows: int, head_dim: int) -> int:
    """Algorithmic bytes of a restore: int8 K,V in + 2-byte K,V scales + 2-byte K,V out."""
    return rows * (6 * head_dim + 4)


def quantize_bytes(rows: int, head_dim: int) -> int:
    """Algorithmic bytes of quantizing K and V: 2-byte in, int8 + 2-byte scale out."""
    return 2 * rows * (3 * head_dim + 2)


def shift_bytes(rows: int, head_dim: int) -> int:
    """Algorithmic bytes of shifting dequantised 16-bit keys: 2-byte in, 2-byte out."""
    return rows * 4 * head_dim


def h2d_bytes(rows: int, head_dim: int) -> int:
    return rows * (2 * head_dim + 4)


def draw_shift(seed: int) -> int:
    return int(np.random.default_rng(seed).integers(1, 4097))


def read_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_profiled_traffic(workload: str) -> float | None:
    """Per-launch DRAM bytes of the workload's dominant kernel, from the committed ncu
    summary (line ``dram_bytes_per_launch_full: <bytes>``); None if not profiled."""
    name = {"llama8b": "dense_restore_llama8b_t8192_ncu.txt",
            "paged": "paged_restore_ragged64_ncu.txt",
            "keyshift": "key_shift_llama8b_t8192_ncu.txt"}.get(workload)
    if name is None:
        return None
    try:
        with open(os.path.join(REPO, "profiles", name)) as f:
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
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=fd, stderr=subprocess.DEVNULL)
            os.close(fd)
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
        if self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        with open(self.path) as f:
            rows = [r.strip().split(",") for r in f if r.strip()]
        os.unlink(self.path)
        sm, smax, reasons, loaded = [], None, set(), []
        for r in rows:
            vals = [v.strip() for v in r]
            try:
                mhz, mx, util = float(vals[1]), float(vals[2]), float(vals[3])
            except (ValueError, IndexError):
                continue
            smax = mx
            sm.append(mhz)
            if util >= 50:
                loaded.append(mhz)
                for name, v in zip(self.NAMES, vals[5:9]):
                    if v.lower() == "active":
                        reasons.add(name)
        pick = loaded or sm
        return {"sm_mhz": statistics.median(pick) if pick else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(loaded)}


def rank_gpus(local_world: int, visible: int, spread: bool = True) -> list[int]:
    """The GPU of each local rank: with more GPUs visible than ranks and ``spread``, rank r
    takes GPU r * (visible // ranks); otherwise GPU r."""
    stride = max(1, visible // max(1, local_world)) if spread else 1
    return [r * stride for r in range(local_world)]


class Dist:
    """One process per GPU (torchrun env); barrier and max-over-ranks over the process
    group (NCCL on GPUs; gloo on CPU for the host-side tests).

    Placement: with more GPUs visible than local ranks, rank r takes GPU r * (visible // ranks)
    (``spread``), so the ranks sit on GPUs that do not share a host link where the machine
    groups its GPUs' links: on these B200 machines GPUs 0-3 share about 115 GB/s of
    host-to-device bandwidth, while four spread GPUs move 213-217 GB/s.  ``spread=False``
    keeps rank r on GPU r."""

    def __init__(self, backend: str = "nccl", spread: bool = True) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.placement = None
        if backend == "nccl":
            local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(self.world)))
            visible = torch.cuda.device_count()
            gpus = rank_gpus(local_world, visible, spread)
            self.device = torch.device("cuda", gpus[self.local])
            self.placement = {"visible_gpus": visible, "gpus": gpus}
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kw = {"device_id": self.device} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def time_steps(fn, steps: int, warmup: int, dist: Dist, per_step_events: bool = False):
    """W untimed steps, then K timed steps bracketed by barrier + synchronize, with one CUDA
    event pair around the K steps on the launching stream; returns (max-over-ranks total ms,
    per-step ms list of this rank).  Per-step ms are total / K unless ``per_step_events`` asks
    for an event after every step (each adds about 3 us between launches on B200, so the
    default measures the steps back to back, as a caller runs them)."""
    stream = torch.cuda.current_stream(dist.device)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dist.device)
    dist.barrier()
    torch.cuda.synchronize(dist.device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(stream)
    for i in range(steps):
        fn()
        if per_step_events or i == steps - 1:
            ev[i + 1].record(stream)
    torch.cuda.synchronize(dist.device)
    dist.barrier()
    total = ev[0].elapsed_time(ev[steps])
    per = ([ev[i].elapsed_time(ev[i + 1]) for i in range(steps)] if per_step_events
           else [total / steps] * steps)
    return dist.max(total), per


# ---------------------------------------------------------------------------------------
# Synthetic inputs
# ---------------------------------------------------------------------------------------
def make_dense_inputs(scb, device, layers, tokens, heads, head_dim, seed, outlier_frac=0.0):
    """Seeded fp16 N(0,1) K/V per layer (optionally a fraction of channels x10),
    quantised on the GPU into [L, T, H, D] codes and [L, T, H, 1] fp16 scales."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    kq = torch.empty((layers, tokens, heads, head_dim), dtype=torch.int8, device=device)
    vq = torch.empty_like(kq)
    ks = torch.empty((layers, tokens, heads, 1), dtype=torch.float16, device=device)
    vs = torch.empty_like(ks)
    n_out = int(round(outlier_frac * head_dim))
    for layer in range(layers):
        for q, s in ((kq, ks), (vq, vs)):
            x = torch.randn((tokens, heads, head_dim), generator=gen, device=device)
            if n_out:
                ch = torch.randperm(head_dim, generator=gen, device=device)[:n_out]
                x[..., ch] *= 10.0
            scb.quantize_kv_int8(x.to(torch.float16), q_out=q[layer], scale_out=s[layer])
    torch.cuda.synchronize(device)
    return kq, ks, vq, vs


def make_paged_case(cfg, seed):
    """Host-side description of the ragged batch: lengths, shifts, shuffled page table."""
    rng = np.random.default_rng(seed)
    n_req, page = cfg["requests"], cfg["page"]
    lens = rng.integers(cfg["min_len"], cfg["max_len"] + 1, n_req).astype(np.int64)
    shifts = rng.integers(0, 4097, n_req).astype(np.float32)
    pages = [(int(n) + page - 1) // page for n in lens]
    n_pool = int(sum(pages))
    perm = rng.permutation(n_pool).astype(np.int32)
    table = np.zeros((n_req, max(pages)), dtype=np.int32)
    k = 0
    for r, n in enumerate(pages):
        table[r, :n] = perm[k:k + n]
        k += n
    return lens, shifts, table, n_pool


# ---------------------------------------------------------------------------------------
# CPU baselines: the reference's own eager functions (speccache/kernels/reference.py, pure
# torch) from the installed copy under baseline/_ref; the oracle (the same arithmetic
# restated on torch-CPU) only when that copy cannot be imported.
# ---------------------------------------------------------------------------------------
REFERENCE_ROOT = os.path.join(REPO, "baseline", "_ref")


def load_reference_kernels():
    """``speccache/kernels/reference.py`` of the installed reference, imported alone (it
    depends on torch only; importing the ``speccache`` package would also build its HTTP app).
    Returns (module, None) or (None, reason)."""
    path = os.path.join(REFERENCE_ROOT, "speccache", "kernels", "reference.py")
    if not os.path.exists(path):
        return None, f"{path} not installed"
    try:
        spec = importlib.util.spec_from_file_location("_speccache_reference_kernels", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as exc:  # reported in the JSON line
        return None, f"import of {path} failed: {exc!r}"


def load_reference_injector():
    """The reference's ``MultiLayerKVInjector`` (its ``apply_rope_shift`` is the key-shift
    workload's reference), imported through the installed ``speccache`` package."""
    if REFERENCE_ROOT not in sys.path:
        sys.path.insert(0, REFERENCE_ROOT)
    import logging

    logging.disable(logging.CRITICAL)
    try:
        from speccache.serving.kv_injector import MultiLayerKVInjector
        return MultiLayerKVInjector, None
    except Exception as exc:
        return None, f"import of speccache.serving.kv_injector failed: {exc!r}"


def _cpu_layer(tokens, heads, head_dim, seed):
    g = torch.Generator().manual_seed(seed)
    kq = torch.randint(-127, 128, (tokens, heads, head_dim), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, (tokens, heads, head_dim), generator=g, dtype=torch.int8)
    ks = (torch.rand((tokens, heads, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)
    vs = (torch.rand((tokens, heads, 1), generator=g) * 0.03 + 1e-3).to(torch.float16)
    return kq, ks, vq, vs


def _restore_fn(ops, kq, ks, vq, vs, dp, head_dim, theta, out_dtype):
    """One restore of one layer: the shift's tables, K dequant + shift, V dequant."""
    if ops["kind"] == "reference":
        ref = ops["mod"]

        def fn():
            c, s = ref.compute_rope_cos_sin_delta(torch.tensor([float(dp)]), head_dim,
                                                  theta_base=theta)
            ref.pytorch_eager_dequant_rope_shift(kq, ks, c, s)
            ref.dequant_value_ref(vq, vs)
        return fn
    oracle = ops["mod"]

    def fn():
        c, s = oracle.compute_rope_cos_sin_delta(dp, head_dim, theta)
        oracle.dequant_rope_shift(kq, ks, c, s, out_dtype=out_dtype)
        oracle.dequant_value(vq, vs, out_dtype=out_dtype)
    return fn


def cpu_ops(workload: str) -> dict:
    """What the CPU legs time: the reference's own functions, else the oracle port."""
    if workload == "keyshift":
        inj, why = load_reference_injector()
        if inj is not None:
            return {"kind": "reference", "mod": inj, "why": None}
    else:
        mod, why = load_reference_kernels()
        if mod is not None:
            return {"kind": "reference", "mod": mod, "why": None}
    return {"kind": "port", "mod": importlib.import_module("oracle.speccache_oracle"), "why": why}


def cpu_step_fn(workload: str, cfg: dict, ops: dict):
    """One bounded CPU sample of the workload; returns (callable, bytes, description)."""
    h, d = cfg["heads"], cfg["head_dim"]
    ref = ops["kind"] == "reference"
    who = ("the reference's own functions (baseline/_ref speccache/kernels/reference.py: "
           "compute_rope_cos_sin_delta, pytorch_eager_dequant_rope_shift, dequant_value_ref"
           + (", quantize_kv_int8" if workload == "roundtrip" else "")
           + "; fp16 outputs, the only dtype they produce, same bytes as bf16)") if ref else (
           "the oracle port (the reference's eager arithmetic restated on torch-CPU)")
    if workload == "paged":
        t = 4224  # the mean request length of the batch
        kq, ks, vq, vs = _cpu_layer(t, h, d, SEED)
        fn = _restore_fn(ops, kq, ks, vq, vs, 2048, d, cfg["theta"], cfg["out"])
        return fn, restore_bytes(t * h, d), (
            f"1 request of mean length {t} of the {cfg['requests']}-request batch "
            f"(H={h}, D={d}, K shift + V dequant) by {who}")
    t = cfg["tokens"]
    if workload == "keyshift":
        g = torch.Generator().manual_seed(SEED)
        k = torch.randn((t, h, d), generator=g).to(torch.float16)
        if ref:
            inj = ops["mod"](1, h, d, device=torch.device("cpu"), max_blocks=1, chunk_size=64)

            def fn():
                inj.apply_rope_shift(k, cfg["delta_p"])
            who = ("the reference's own MultiLayerKVInjector.apply_rope_shift "
                   "(speccache/serving/kv_injector.py:246-283, theta 10000: it takes no theta)")
        else:
            oracle = ops["mod"]

            def fn():
                oracle.apply_rope_shift(k, cfg["delta_p"], cfg["theta"])
        return fn, shift_bytes(t * h, d), (
            f"1 of {cfg['layers']} layers (T={t}, H={h}, D={d}: RoPE shift of fp16 keys) by {who}")
    if workload == "roundtrip":
        g = torch.Generator().manual_seed(SEED)
        xk = torch.randn((t, h, d), generator=g).to(torch.float16)
        xv = torch.randn((t, h, d), generator=g).to(torch.float16)
        mod = ops["mod"]

        def fn():
            kq, ks = mod.quantize_kv_int8(xk)
            vq, vs = mod.quantize_kv_int8(xv)
            _restore_fn(ops, kq, ks, vq, vs, cfg["delta_p"], d, cfg["theta"], cfg["out"])()

        return fn, quantize_bytes(t * h, d) + restore_bytes(t * h, d), (
            f"1 of {cfg['layers']} layers (T={t}, H={h}, D={d}: quantize K,V then restore) by {who}")
    kq, ks, vq, vs = _cpu_layer(t, h, d, SEED)
    dp = cfg.get("delta_p", draw_shift(SEED))
    fn = _restore_fn(ops, kq, ks, vq, vs, dp, d, cfg["theta"], cfg["out"])
    return fn, restore_bytes(t * h, d), (
        f"1 of {cfg['layers']} layers (T={t}, H={h}, D={d}, K shift + V dequant) by {who}")


def cpu_baseline(workload: str, cfg: dict, time_limit_s: float = 10.0) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    ops = cpu_ops(workload)
    fn, nbytes, what = cpu_step_fn(workload, cfg, ops)
    fn()  # first call outside the timing (allocator warm-up)
    times = []
    t_end = time.perf_counter() + time_limit_s
    while len(times) < 5 or (time.perf_counter() < t_end and len(times) < 200):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    out = {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
           "kind": ops["kind"], "sample": f"{what}; median of {len(times)} runs; per-layer cost "
                                          "is independent of the layer, so it scales linearly"}
    if ops["why"]:
        out["reference_unavailable"] = ops["why"]
    return out


def run_reference(args) -> None:
    """The reference's CPU implementation of the path (its own eager functions from
    baseline/_ref, else the oracle port) on the host cores; rank 0 only under torchrun."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = WORKLOADS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    ops = cpu_ops(args.workload)
    fn, nbytes, what = cpu_step_fn(args.workload, cfg, ops)
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    mean = sum(times) / len(times)
    value = nbytes / mean / 1e9
    base = {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": ops["kind"],
            "sample": f"{what}, one per step"}
    if ops["why"]:
        base["reference_unavailable"] = ops["why"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8/fp16 in, fp32 math, 16-bit out", "data": "synthetic (seeded)",
        "config": workload_config(args.workload, cfg, world),
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = ("dequant+RoPE-shift GB/s (algorithmic bytes) & % of B200 HBM peak; "
          "T=8192 KV restore ms")


def workload_config(workload: str, cfg: dict, world: int, gather: bool = False) -> dict:
    if workload == "llama8b":
        return {"workload": "llama3-8b KV restore: 32 layers x (K,V), T=8192, 8 KV heads x 128 "
                            "per GPU, theta=5e5, one delta_p in [1,4096], bf16 per-layer caches",
                "layers": cfg["layers"], "seq_len": cfg["tokens"], "kv_heads_per_gpu": cfg["heads"],
                "head_dim": cfg["head_dim"], "delta_p": draw_shift(SEED), "theta": cfg["theta"],
                "parallelism": f"kv-head shards x{world} (weak)",
                "l2": "inputs+outputs 1.62 GB per step > 126 MB L2 (no flush needed)"}
    if workload == "paged":
        return {"workload": "ragged paged batch: 64 requests, lengths U[256,8192], delta_p "
                            "U[0,4096], 64-token pages, shuffled page table, H=8, D=128, "
                            "bf16 packed caches", "requests": cfg["requests"], "page": cfg["page"],
                "kv_heads": cfg["heads"], "head_dim": cfg["head_dim"], "theta": cfg["theta"],
                "parallelism": f"independent batches x{world} (weak)",
                "l2": "about 1.7 GB per step > L2 (no flush needed)"}
    if workload == "roundtrip":
        return {"workload": "qwen2.5-7b-like round trip: 28 layers, T=16384, 4 KV heads x 128, "
                            "theta=1e6, 2% outlier channels; quantize then restore (delta_p 2048) "
                            "to fp16", "layers": cfg["layers"], "seq_len": cfg["tokens"],
                "kv_heads": cfg["heads"], "head_dim": cfg["head_dim"], "theta": cfg["theta"],
                "delta_p": cfg["delta_p"], "parallelism": f"replicas x{world} (weak)",
                "l2": "3.4 GB per step > L2 (no flush needed)"}
    if workload == "keyshift":
        return {"workload": "llama3-8b key shift: dequantised fp16 keys of 32 layers, T=8192, "
                            "8 KV heads x 128, delta_p -384, theta=5e5 (the injector's "
                            "apply_rope_shift), one launch", "layers": cfg["layers"],
                "seq_len": cfg["tokens"], "kv_heads": cfg["heads"], "head_dim": cfg["head_dim"],
                "delta_p": cfg["delta_p"], "theta": cfg["theta"],
                "parallelism": f"replicas x{world} (weak)",
                "l2": "1.07 GB per step > L2 (no flush needed)"}
    return {"workload": "llama3-70b KV restore from pinned host: 80 layers, T=32768, 8 KV heads "
                        "x 128 sharded over the GPUs, delta_p 8192, theta=5e5, bf16"
                        + ("; all heads gathered on GPU 0" if gather else ""),
            "layers": cfg["layers"], "seq_len": cfg["tokens"], "kv_heads_total": cfg["heads"],
            "kv_heads_per_gpu": cfg["heads"] // world, "head_dim": cfg["head_dim"],
            "parallelism": f"kv-head shards x{world} (strong)", "l2": "pinned host source"}


# ---------------------------------------------------------------------------------------
# GPU arms
# ---------------------------------------------------------------------------------------
def roofline(nbytes: float, per_step_ms: list[float], workload: str) -> dict:
    peak, kind = read_peaks()
    avg = sum(per_step_ms) / len(per_step_ms)
    achieved = nbytes / (avg / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "traffic": read_profiled_traffic(workload),
            "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)",
            "launch_ms": avg}


def e2e_line(nbytes, e2e_ms, steps, world, h2d, d2h, launches, path, extra=None) -> dict:
    out = {"value": nbytes * world * steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
           "restore_ms": e2e_ms / steps, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h),
           "h2d_gbs": h2d * world * steps / (e2e_ms / 1e3) / 1e9,
           "h2d_gbs_per_gpu": h2d * steps / (e2e_ms / 1e3) / 1e9, "path": path,
           "gpu_launches": launches}
    out.update(extra or {})
    return out


def bench_llama8b(args, scb, dist: Dist, cfg: dict):
    from speccache_b200.cache import KVRestorePipeline

    layers, t, h, d = args.layers, cfg["tokens"], cfg["heads"], cfg["head_dim"]
    dev, dp, theta = dist.device, draw_shift(SEED), cfg["theta"]
    kq, ks, vq, vs = make_dense_inputs(scb, dev, layers, t, h, d, SEED + 1000 * dist.rank)
    k_out = torch.empty((layers, t, h, d), dtype=cfg["out"], device=dev)
    v_out = torch.empty_like(k_out)
    nbytes = restore_bytes(layers * t * h, d)

    def step():
        scb.restore_layers(kq, ks, vq, vs, delta_p=dp, theta=theta, k_out=k_out, v_out=v_out)

    total_ms, per = time_steps(step, args.steps, args.warmup, dist)
    line = {"value": nbytes * dist.world * args.steps / (total_ms / 1e3) / 1e9,
            "ms_per_step": total_ms / args.steps, "roofline": roofline(nbytes, per, "llama8b"),
            "gpu_launches": args.steps}
    if args.skip_e2e:
        return line
    n_blocks = t // CHUNK
    scattered = args.block_order == "scattered"
    slab_blocks = 2 * n_blocks if scattered else n_blocks
    if scattered:  # block i of the restore lives at slab block ids[i]: every block its own run
        ids = [2 * b + 1 for b in range(n_blocks)]
        random.Random(SEED).shuffle(ids)
    else:
        ids = list(range(n_blocks))
    with KVRestorePipeline(layers, slab_blocks, CHUNK, h, d, device=dev, n_slots=3,
                           max_restore_blocks=n_blocks, write_combined=args.write_combined) as pipe:
        where = torch.tensor(ids)
        for slab, src, last in ((pipe.k_quant, kq, d), (pipe.v_quant, vq, d),
                                (pipe.k_scale, ks, 1), (pipe.v_scale, vs, 1)):
            slab[:, where] = src.cpu().view(layers, n_blocks, CHUNK, h, last)
        ko = [k_out[i] for i in range(layers)]
        vo = [v_out[i] for i in range(layers)]
        shifts = [dp] * n_blocks
        tail = torch.empty((2, h, d), dtype=cfg["out"]).pin_memory()

        def e2e_step():
            pipe.restore(ids, shifts, ko, vo, theta=theta)
            tail[0].copy_(k_out[layers - 1, t - 1], non_blocking=True)
            tail[1].copy_(v_out[layers - 1, t - 1], non_blocking=True)

        e2e_ms, _ = time_steps(e2e_step, args.steps, args.warmup, dist)
        launches, copies = pipe.restore_plan(ids)
        runs = 1 + sum(1 for a, b in zip(ids, ids[1:]) if b != a + 1)
        ceiling = h2d_ceiling(pipe, dist, sustained_steps=args.steps)
        # one restore on its own (latency, nothing overlapping it)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        single_ms = e0.elapsed_time(e1)
        status = pipe.status()
    line["e2e"] = e2e_line(nbytes, e2e_ms, args.steps, dist.world, h2d_bytes(layers * t * h, d),
                           tail.numel() * tail.element_size(), launches * args.steps,
                           f"sc_pipeline_restore from pinned host slabs, {launches} kernel "
                           f"launches per restore of {layers} layers",
                           {"restore_ms_single": single_ms, "device_status": status,
                            "block_order": args.block_order, "runs": runs,
                            "copies_per_restore": copies})
    line["e2e"].update(ceiling)
    line["e2e"]["h2d_vs_ceiling"] = line["e2e"]["h2d_gbs"] / ceiling["h2d_ceiling_gbs"]
    line["e2e"]["h2d_vs_sustained_ceiling"] = (line["e2e"]["h2d_gbs"] /
                                               ceiling["h2d_ceiling_sustained_gbs"])
    return line


def h2d_ceiling(pipe, dist: Dist, reps: int = 5, sustained_steps: int = 20) -> dict:
    """Copy-only ceiling of the host-to-device leg at this N: every rank copies its whole
    pinned slab (the K and V codes and scales of every layer, the bytes one restore moves)
    into HBM with one cudaMemcpyAsync per slab and nothing else running, all ranks at once
    between barriers.  Each rep is timed on every rank with CUDA events; a rep's time is the
    slowest rank's, and the ceiling is the best rep (PCIe links on a shared machine see
    other jobs' traffic, so single reps vary).  The sustained ceiling copies the slab
    ``sustained_steps`` times back to back, as the timed restores run, for hosts whose
    transfer rate drops over a longer stream."""
    slabs = [pipe.k_quant, pipe.v_quant, pipe.k_scale, pipe.v_scale]
    srcs = [x.reshape(-1).view(torch.uint8) for x in slabs]
    nbytes = sum(x.numel() for x in srcs)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dist.device)
    parts = []
    off = 0
    for x in srcs:
        parts.append(dst[off:off + x.numel()])
        off += x.numel()

    def copy_all():
        for d_, s_ in zip(parts, srcs):
            d_.copy_(s_, non_blocking=True)

    copy_all()  # warm-up (first touch of the destination)
    times = []
    for _ in range(reps):
        ms, _ = time_steps(copy_all, 1, 0, dist)
        times.append(ms)
    sustained_ms, _ = time_steps(copy_all, sustained_steps, 1, dist)
    del dst
    best = min(times)
    return {"h2d_ceiling_gbs": nbytes * dist.world / (best / 1e3) / 1e9,
            "h2d_ceiling_ms": best, "h2d_ceiling_reps_ms": times,
            "h2d_ceiling_sustained_gbs":
                nbytes * dist.world * sustained_steps / (sustained_ms / 1e3) / 1e9,
            "h2d_ceiling_sustained_ms": sustained_ms / sustained_steps,
            "h2d_ceiling_how": f"{len(srcs)} cudaMemcpyAsync of the rank's pinned slabs "
                               f"({nbytes} B) into HBM per rank, all ranks at once between "
                               f"barriers, nothing else running; best of {reps} reps"}


def gather_check(scb, dist: Dist, layers: int = 3, blocks: int = 6, chunk: int = 64,
                 heads: int = 8, head_dim: int = 128, theta: float = 500000.0) -> dict:
    """The head-shard gather onto one GPU, checked in the run (N >= 2, outside the timing).

    Every rank restores its KV-head shard of a small model (3 layers x 4 blocks of 64
    tokens, 8 heads, per-block shifts) from its own pinned slab straight into GPU 0's caches
    (HeadShardGather: CUDA IPC mapping, plain 32-byte peer stores from the restore kernel;
    no multicast, no TMA, no library kernel on peer memory).  GPU 0 then restores every
    head itself with the dense kernel (sc_dequant_rope_kv, a different kernel on the same
    arithmetic) and compares all K and V bits."""
    from speccache_b200.cache import HeadShardGather, KVRestorePipeline, shard_view

    ids, shifts = [4, 0, 1, 5], [-300, 12, 12, 4000]
    g = torch.Generator().manual_seed(4242)  # the whole model's codes, the same on every rank
    kq = torch.randint(-127, 128, (layers, blocks, chunk, heads, head_dim), generator=g,
                       dtype=torch.int8)
    vq = torch.randint(-127, 128, kq.shape, generator=g, dtype=torch.int8)
    ks = (torch.rand(kq.shape[:4] + (1,), generator=g) * 0.05 + 1e-3).half()
    vs = (torch.rand(kq.shape[:4] + (1,), generator=g) * 0.05 + 1e-3).half()
    world, rank, dev = dist.world, dist.rank, dist.device
    n_tok = len(ids) * chunk
    out = {"layers": layers, "tokens": n_tok, "heads": heads, "heads_per_rank": heads // world,
           "owner": 0}
    with KVRestorePipeline(layers, blocks, chunk, heads // world, head_dim, device=dev) as pipe:
        for dst, src in ((pipe.k_quant, kq), (pipe.k_scale, ks), (pipe.v_quant, vq),
                         (pipe.v_scale, vs)):
            dst.copy_(shard_view(src, heads, world, rank, 3))
        k_full = v_full = None
        if rank == 0:
            k_full = torch.zeros((layers, n_tok, heads, head_dim), dtype=torch.bfloat16, device=dev)
            v_full = torch.zeros_like(k_full)
        gather = HeadShardGather(pipe, k_full, v_full, owner=0, rank=rank, world_size=world,
                                 num_kv_heads=heads)
        gather.restore(ids, shifts, theta=theta)
        pipe.synchronize()
        out["device_status_max"] = int(dist.max(float(pipe.status())))
        dist.barrier()  # every writer's stream has completed
        if rank == 0:
            exp_k = torch.empty_like(k_full)
            exp_v = torch.empty_like(v_full)
            for i, (b, dp) in enumerate(zip(ids, shifts)):
                sl = slice(i * chunk, (i + 1) * chunk)
                scb.restore_layers(kq[:, b].to(dev), ks[:, b].to(dev), vq[:, b].to(dev),
                                   vs[:, b].to(dev), delta_p=dp, theta=theta,
                                   k_out=exp_k[:, sl], v_out=exp_v[:, sl])
            torch.cuda.synchronize(dev)
            out["k_mismatched"] = int((k_full.view(torch.int16) != exp_k.view(torch.int16)).sum())
            out["v_mismatched"] = int((v_full.view(torch.int16) != exp_v.view(torch.int16)).sum())
            out["ok"] = (out["k_mismatched"] == 0 and out["v_mismatched"] == 0
                         and out["device_status_max"] == 0)
        dist.barrier()  # the other ranks keep their mappings until GPU 0 has checked
        gather.close()
    return out


def bench_paged(args, scb, dist: Dist, cfg: dict):
    dev = dist.device
    h, d, page = cfg["heads"], cfg["head_dim"], cfg["page"]
    lens, shifts, table, n_pool = make_paged_case(cfg, SEED + dist.rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + dist.rank)
    pkq = torch.randint(-127, 128, (n_pool, page, h, d), generator=gen, device=dev, dtype=torch.int8)
    pvq = torch.randint(-127, 128, (n_pool, page, h, d), generator=gen, device=dev, dtype=torch.int8)
    pks = (torch.rand((n_pool, page, h, 1), generator=gen, device=dev) * 0.03 + 1e-3).half()
    pvs = (torch.rand((n_pool, page, h, 1), generator=gen, device=dev) * 0.03 + 1e-3).half()
    total = int(lens.sum())
    k_out = torch.empty((total, h, d), dtype=cfg["out"], device=dev)
    v_out = torch.empty_like(k_out)
    cu = np.concatenate([[0], np.cumsum(lens)])
    offs = torch.from_numpy(cu[:-1] * h * d).to(dev)
    tab, lens_d = torch.from_numpy(table).to(dev), torch.from_numpy(lens.astype(np.int32)).to(dev)
    dps = torch.from_numpy(shifts).to(dev)
    nbytes = restore_bytes(total * h, d)

    def step():
        scb.restore_paged(pkq, pks, pvq, pvs, tab, lens_d, dps, theta=cfg["theta"],
                          k_out=k_out, v_out=v_out, out_offsets=offs)

    total_ms, per = time_steps(step, args.steps, args.warmup, dist)
    status = scb.paged_status(dev)
    line = {"value": nbytes * dist.world * args.steps / (total_ms / 1e3) / 1e9,
            "ms_per_step": total_ms / args.steps, "roofline": roofline(nbytes, per, "paged"),
            "gpu_launches": args.steps, "device_status": status,
            "tokens": total, "pool_pages": n_pool}
    if args.skip_e2e:
        return line
    # e2e: the pool's pages arrive from pinned host memory, then one restore launch
    hosts = [x.cpu().pin_memory() for x in (pkq, pks, pvq, pvs)]
    tail = torch.empty((2, h, d), dtype=cfg["out"]).pin_memory()

    def e2e_step():
        for dst, src in zip((pkq, pks, pvq, pvs), hosts):
            dst.copy_(src, non_blocking=True)
        step()
        tail[0].copy_(k_out[total - 1], non_blocking=True)
        tail[1].copy_(v_out[total - 1], non_blocking=True)

    e2e_ms, _ = time_steps(e2e_step, args.steps, args.warmup, dist)
    h2d = sum(x.numel() * x.element_size() for x in hosts)
    line["e2e"] = e2e_line(nbytes, e2e_ms, args.steps, dist.world, h2d,
                           tail.numel() * tail.element_size(), args.steps,
                           "pool pages H2D from pinned host, then sc_restore_paged")
    return line


def bench_roundtrip(args, scb, dist: Dist, cfg: dict):
    dev = dist.device
    layers, t, h, d = cfg["layers"], cfg["tokens"], cfg["heads"], cfg["head_dim"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + dist.rank)
    xs = []
    for _ in range(2):
        x = torch.randn((layers, t, h, d), generator=gen, device=dev)
        ch = torch.randperm(d, generator=gen, device=dev)[: max(1, round(0.02 * d))]
        x[..., ch] *= 10.0
        xs.append(x.to(torch.float16).view(layers * t, h, d))
    xk, xv = xs
    kq = torch.empty((layers * t, h, d), dtype=torch.int8, device=dev)
    vq = torch.empty_like(kq)
    ks = torch.empty((layers * t, h, 1), dtype=torch.float16, device=dev)
    vs = torch.empty_like(ks)
    k_out = torch.empty((layers, t, h, d), dtype=cfg["out"], device=dev)
    v_out = torch.empty_like(k_out)
    rows = layers * t * h
    nbytes = quantize_bytes(rows, d) + restore_bytes(rows, d)

    def step():
        scb.quantize_kv_int8(xk, q_out=kq, scale_out=ks)
        scb.quantize_kv_int8(xv, q_out=vq, scale_out=vs)
        scb.restore_layers(kq.view(layers, t, h, d), ks.view(layers, t, h, 1),
                           vq.view(layers, t, h, d), vs.view(layers, t, h, 1),
                           delta_p=cfg["delta_p"], theta=cfg["theta"], k_out=k_out, v_out=v_out)

    total_ms, per = time_steps(step, args.steps, args.warmup, dist)
    line = {"value": nbytes * dist.world * args.steps / (total_ms / 1e3) / 1e9,
            "ms_per_step": total_ms / args.steps, "roofline": roofline(nbytes, per, "roundtrip"),
            "gpu_launches": 3 * args.steps}
    if args.skip_e2e:
        return line
    hk, hv = xk.cpu().pin_memory(), xv.cpu().pin_memory()
    tail = torch.empty((2, h, d), dtype=cfg["out"]).pin_memory()

    def e2e_step():
        xk.copy_(hk, non_blocking=True)
        xv.copy_(hv, non_blocking=True)
        step()
        tail[0].copy_(k_out[layers - 1, t - 1], non_blocking=True)
        tail[1].copy_(v_out[layers - 1, t - 1], non_blocking=True)

    e2e_ms, _ = time_steps(e2e_step, args.steps, args.warmup, dist)
    line["e2e"] = e2e_line(nbytes, e2e_ms, args.steps, dist.world,
                           2 * hk.numel() * hk.element_size(), tail.numel() * tail.element_size(),
                           3 * args.steps, "fp16 K/V H2D from pinned host, quantize, restore")
    line["offload"] = offload_line(args, dist, xk.view(layers, t, h, d), xv.view(layers, t, h, d))
    return line


def offload_line(args, dist: Dist, xk: torch.Tensor, xv: torch.Tensor) -> dict:
    """The cold-miss direction: every layer's fp16 K/V quantized on the GPU and moved into
    the pinned host slabs (sc_pipeline_offload), timed on the current stream through
    sc_pipeline_join (no host wait inside the step).  With ``--block-order scattered`` the
    blocks go to every other block of a slab twice as large, in a seeded random order (every
    block its own run), as a pool that allocates blocks from a free list would place them."""
    from speccache_b200.cache import KVRestorePipeline

    layers, t, h, d = xk.shape
    n_blocks = t // CHUNK
    scattered = args.block_order == "scattered"
    if scattered:
        ids = [2 * b + 1 for b in range(n_blocks)]
        random.Random(SEED).shuffle(ids)
    else:
        ids = list(range(n_blocks))
    with KVRestorePipeline(layers, 2 * n_blocks if scattered else n_blocks, CHUNK, h, d,
                           device=dist.device, max_restore_blocks=n_blocks) as pipe:
        def step():
            for layer in range(layers):
                pipe.offload(layer, ids, xk[layer], xv[layer])
            pipe.join()

        ms, _ = time_steps(step, args.steps, args.warmup, dist)
        status = pipe.status()
        per_layer, copies = pipe.offload_plan(ids)  # launches and copy commands per layer
    rows = layers * t * h
    d2h = 2 * rows * (d + 2)  # int8 codes and fp16 scales of K and V
    return {"ms_per_step": ms / args.steps,
            "d2h_gbs": d2h * dist.world * args.steps / (ms / 1e3) / 1e9,
            "quantize_gbs": quantize_bytes(rows, d) * dist.world * args.steps / (ms / 1e3) / 1e9,
            "d2h_bytes_per_step": d2h, "gpu_launches": per_layer * layers * args.steps,
            "copies_per_step": copies * layers, "block_order": args.block_order,
            "device_status": status,
            "path": ("quantize on the GPU into a staging slot, one scatter kernel per layer "
                     "writing the blocks into the mapped pinned slabs" if scattered else
                     "quantize on the GPU into a staging slot, 2-D D2H copies into the pinned "
                     "slabs")}


def bench_keyshift(args, scb, dist: Dist, cfg: dict):
    layers = args.layers if args.layers != WORKLOADS["llama8b"]["layers"] else cfg["layers"]
    t, h, d = cfg["tokens"], cfg["heads"], cfg["head_dim"]
    gen = torch.Generator(device=dist.device)
    gen.manual_seed(SEED + dist.rank)
    k = torch.randn((layers * t, h, d), generator=gen, device=dist.device).to(torch.float16)
    out = torch.empty_like(k)
    rows = layers * t * h
    nbytes = shift_bytes(rows, d)

    def step():
        scb.rope_shift_keys(k, cfg["delta_p"], theta=cfg["theta"], out=out)

    total_ms, per = time_steps(step, args.steps, args.warmup, dist)
    line = {"value": nbytes * dist.world * args.steps / (total_ms / 1e3) / 1e9,
            "ms_per_step": total_ms / args.steps, "roofline": roofline(nbytes, per, "keyshift"),
            "gpu_launches": args.steps}
    if args.skip_e2e:
        return line
    hk = k.cpu().pin_memory()
    tail = torch.empty((1, h, d), dtype=torch.float16).pin_memory()

    def e2e_step():
        k.copy_(hk, non_blocking=True)
        step()
        tail.copy_(out[-1:], non_blocking=True)

    e2e_ms, _ = time_steps(e2e_step, args.steps, args.warmup, dist)
    line["e2e"] = e2e_line(nbytes, e2e_ms, args.steps, dist.world, hk.numel() * hk.element_size(),
                           tail.numel() * tail.element_size(), args.steps,
                           "fp16 keys H2D from pinned host, then sc_rope_shift_keys")
    return line


def bench_llama70b(args, scb, dist: Dist, cfg: dict):
    from speccache_b200.cache import HeadShardGather, KVRestorePipeline

    dev = dist.device
    layers, t, d = cfg["layers"], cfg["tokens"], cfg["head_dim"]
    if cfg["heads"] % dist.world:
        raise SystemExit(f"{cfg['heads']} KV heads do not split over {dist.world} GPUs")
    h = cfg["heads"] // dist.world
    n_blocks = t // CHUNK
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + dist.rank)
    rows = layers * t * h
    nbytes = restore_bytes(rows, d)
    gather = None
    k_out = v_out = None
    if args.gather:
        # all heads land on GPU 0: its full caches, written by every rank's kernels
        if dist.rank == 0:
            k_out = torch.empty((layers, t, cfg["heads"], d), dtype=cfg["out"], device=dev)
            v_out = torch.empty_like(k_out)
    else:
        k_out = torch.empty((layers, t, h, d), dtype=cfg["out"], device=dev)
        v_out = torch.empty_like(k_out)
    with KVRestorePipeline(layers, n_blocks, CHUNK, h, d, device=dev, n_slots=3,
                           write_combined=args.write_combined) as pipe:
        for layer in range(layers):  # this rank's head shard of every layer
            for q, s in ((pipe.k_quant, pipe.k_scale), (pipe.v_quant, pipe.v_scale)):
                x = torch.randn((t, h, d), generator=gen, device=dev).to(torch.float16)
                qd, sd = scb.quantize_kv_int8(x)
                q[layer].view(t, h, d).copy_(qd.cpu())
                s[layer].view(t, h, 1).copy_(sd.cpu())
        ids, shifts = list(range(n_blocks)), [cfg["delta_p"]] * n_blocks
        if args.gather:
            gather = HeadShardGather(pipe, k_out, v_out, owner=0, rank=dist.rank,
                                     world_size=dist.world, num_kv_heads=cfg["heads"])
        else:
            ko = [k_out[i] for i in range(layers)]
            vo = [v_out[i] for i in range(layers)]
        tail = torch.empty((2, h, d), dtype=cfg["out"]).pin_memory()

        def step():
            if gather is not None:
                gather.restore(ids, shifts, theta=cfg["theta"])
            else:
                pipe.restore(ids, shifts, ko, vo, theta=cfg["theta"])
            if k_out is not None:
                tail[0].copy_(k_out[layers - 1, t - 1, :h], non_blocking=True)
                tail[1].copy_(v_out[layers - 1, t - 1, :h], non_blocking=True)

        total_ms, _ = time_steps(step, args.steps, args.warmup, dist)
        status = pipe.status()
        launches, copies = pipe.restore_plan(ids)
        if gather is not None:
            dist.barrier()  # the owner's buffers stay alive until every writer is done
            gather.close()
    h2d = h2d_bytes(rows, d)
    path = ("each rank's kernels store its head shard into GPU 0's caches over NVLink"
            if args.gather else "sc_pipeline_restore from pinned host slabs (bytes of all ranks)")
    e2e = e2e_line(nbytes, total_ms, args.steps, dist.world, h2d,
                   tail.numel() * tail.element_size() if k_out is not None else 0,
                   launches * args.steps, path,
                   {"device_status": status, "copies_per_restore": copies})
    return {"value": e2e["value"], "ms_per_step": total_ms / args.steps, "scaling": "strong",
            "gpu_launches": launches * args.steps, "e2e": e2e,
            "roofline": {"bound": "pcie-h2d", "achieved": e2e["h2d_gbs"] / dist.world,
                         "unit": "GB/s per GPU", "peak": None, "frac": None, "traffic": None}}


def run_ours(args) -> None:
    dist = Dist(spread=not args.pack_ranks)
    scb = importlib.import_module("intelligent-bell_b200")
    cfg = WORKLOADS[args.workload]
    fn = {"llama8b": bench_llama8b, "paged": bench_paged, "roundtrip": bench_roundtrip,
          "llama70b": bench_llama70b, "keyshift": bench_keyshift}[args.workload]
    with ClockSampler(dist.device.index or 0) as clocks:
        part = fn(args, scb, dist, cfg)
    check = None
    if dist.world > 1 and args.workload in ("llama8b", "llama70b") and not args.skip_gather_check:
        check = gather_check(scb, dist)
        part["gather_check"] = check
    if dist.rank == 0:
        line = {"metric": METRIC, "value": part.pop("value"), "unit": "GB/s",
                "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": part.pop("ms_per_step"), "higher_is_better": True,
                "scaling": part.pop("scaling", "weak"), "vs_baseline": None,
                "dtype": ("fp16" if args.workload == "keyshift" else "int8") + " in, fp32 math, "
                         + str(cfg["out"]).replace("torch.", "") + " out",
                "data": "synthetic: seeded, see config",
                "config": workload_config(args.workload, cfg, dist.world, args.gather)}
        if dist.world > 1:
            line["config"]["placement"] = dist.placement
        line.update(part)
        line["clocks"] = clocks.summary()
        if dist.world == 1 and not args.skip_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.workload, cfg)
        print(json.dumps(line), flush=True)
    dist.close()
    if check is not None and dist.rank == 0 and not check.get("ok", False):
        raise SystemExit(f"head-shard gather check failed: {check}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama8b")
    ap.add_argument("--layers", type=int, default=WORKLOADS["llama8b"]["layers"],
                    help="llama8b / keyshift layers per step (32 = the workload; fewer only "
                         "for profiling captures)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling aid: kernel leg only")
    ap.add_argument("--skip-cpu-baseline", action="store_true", help="profiling aid")
    ap.add_argument("--write-combined", action="store_true",
                    help="pin the host slabs write-combined (pipeline workloads)")
    ap.add_argument("--pack-ranks", action="store_true",
                    help="N > 1: rank r on GPU r even when more GPUs are visible (default: "
                         "spread the ranks over the visible GPUs)")
    ap.add_argument("--skip-gather-check", action="store_true",
                    help="N > 1: skip the in-run check of the head-shard gather onto GPU 0")
    ap.add_argument("--gather", action="store_true",
                    help="llama70b: restore every rank's head shard into GPU 0's caches (NVLink)")
    ap.add_argument("--block-order", choices=["contiguous", "scattered"], default="contiguous",
                    help="llama8b e2e restore and roundtrip offload: consecutive blocks "
                         "(default), or the same number of blocks scattered over a slab twice "
                         "as large (every other block, in a seeded random order: every block "
                         "its own run)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
