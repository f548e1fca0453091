"""Failure handling and stream ordering of the restore pipeline, with the failures made on
the host (nothing here faults, traps or hangs the GPU):

* a pinned-allocation failure (host failpoint ``SC_FAILPOINT_HOST_ALLOC``) is reported as an
  error, cleans up what was allocated, and leaves the library usable;
* a stalled stream (torch's bounded ``_sleep`` kernel ahead of the restores) does not block the
  enqueue (the pipeline loads its kernels at creation) and makes
  ``synchronize`` with a short deadline raise ``TimeoutError``; a later wait completes and the
  results are right;
* ``preload()`` loads every kernel up front, so a fresh process's first calls enqueued behind
  running work do not wait for it;
* stream hazards: back-to-back restores and offloads that reuse the staging slots (on the
  single-stage, block-stage and layer-by-layer paths), the shift metadata and the offload slots,
  with random GPU-side delays on the compute stream and random host delays between enqueues,
  all checked against the oracle.
"""

from __future__ import annotations

import os
import random
import time

import pytest
import torch

from conftest import bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
CYCLES_PER_MS = 2_000_000  # the sleep kernel counts SM clock cycles (about 2 GHz)


def _fill(pipe, seed):
    g = torch.Generator().manual_seed(seed)
    for t in (pipe.k_quant, pipe.v_quant):
        t.copy_(torch.randint(-127, 128, tuple(t.shape), generator=g, dtype=torch.int8))
    for t in (pipe.k_scale, pipe.v_scale):
        t.copy_((torch.rand(tuple(t.shape), generator=g) * 0.05 + 1e-3).half())


def _check_layers(oracle, pipe, k_out, v_out, ids, dps, theta=10000.0):
    for layer in range(pipe.num_layers):
        kr, vr = oracle.restore_blocks(pipe.k_quant[layer], pipe.k_scale[layer], pipe.v_quant[layer],
                                       pipe.v_scale[layer], ids, dps, theta, k_out[layer].dtype)
        torch.testing.assert_close(k_out[layer].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(v_out[layer].cpu(), vr), layer


@pytest.mark.parametrize("fail_at", [1, 2, 3])
def test_pinned_allocation_failure_is_reported_and_cleaned_up(scb, fail_at):
    from speccache_b200.cache import KVRestorePipeline

    os.environ["SC_FAILPOINT_HOST_ALLOC"] = str(fail_at)
    try:
        with pytest.raises(RuntimeError, match="cudaHostAlloc"):
            KVRestorePipeline(2, 4, 16, 2, 128, device=DEV)
    finally:
        del os.environ["SC_FAILPOINT_HOST_ALLOC"]
    with KVRestorePipeline(2, 4, 16, 2, 128, device=DEV) as pipe:  # the library still works
        assert pipe.k_quant.shape == (2, 4, 16, 2, 128)


@pytest.mark.parametrize("per_layer", [False, True])
def test_synchronize_times_out_on_a_stalled_stream(scb, oracle, per_layer):
    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, chunk, h, d = 3, 6, 32, 4, 128
    with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, per_layer=per_layer) as pipe:
        _fill(pipe, 3)
        cases = [([5, 0, 1], [-50, 7, 7]), ([2], [300]), ([3, 4], [0, -9]), ([1, 5, 2], [4, 4, 4])]
        outs = []
        for ids, _ in cases:
            k_out = torch.empty((layers, len(ids) * chunk, h, d), dtype=torch.bfloat16, device=DEV)
            outs.append((k_out, torch.empty_like(k_out)))
        torch.cuda._sleep(1000 * CYCLES_PER_MS)  # about one second of bounded delay
        # The pipeline loaded its kernels when it was created, so restores are enqueued
        # without waiting for the device (a lazy module load at the first launch would block
        # until the delay is over); four restores in flight use distinct host metadata
        # buffers, so none of them waits for the delayed kernels either.
        for (ids, dps), (k_out, v_out) in zip(cases, outs):
            t0 = time.perf_counter()
            pipe.restore(ids, dps, list(k_out), list(v_out))
            assert time.perf_counter() - t0 < 0.3
        with pytest.raises(TimeoutError):
            pipe.synchronize(timeout=0.05)
        pipe.synchronize(timeout=60.0)
        assert pipe.status() == 0
        for (ids, dps), (k_out, v_out) in zip(cases, outs):
            _check_layers(oracle, pipe, k_out, v_out, ids, dps)


PRELOAD_SCRIPT = r"""
import importlib, sys, time, torch
sys.path.insert(0, sys.argv[1])
scb = importlib.import_module("intelligent-bell_b200")
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
x = torch.randn((64, 8, 128), device=dev).half()
torch.cuda.synchronize()
scb.preload()
torch.cuda._sleep(1_000_000_000)  # about half a second of bounded delay
t0 = time.perf_counter()
q, s = scb.quantize_kv_int8(x)
scb.restore_layers(q[None], s[None], q[None], s[None], delta_p=3)
scb.dequant_kv_cache(q, s, q, s, delta_p=7)
scb.rope_shift_keys(x, 5)
dt = time.perf_counter() - t0
torch.cuda.synchronize()
print(f"first calls enqueued in {dt:.4f} s")
"""


def test_preloaded_first_calls_do_not_wait_for_the_device(scb):
    # a fresh process: its first launches of the library's kernels come after the preload
    import subprocess
    import sys

    from conftest import REPO

    out = subprocess.run([sys.executable, "-c", PRELOAD_SCRIPT, REPO], capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    dt = float(out.stdout.strip().split()[-2])
    assert dt < 0.25, out.stdout


# The restore paths: small restores in one stage and one launch, larger ones in block stages
# (here 90-98 blocks of 64 tokens x 8 heads over 6 layers, 85 blocks per stage: stages of
# 44-49, 44-48 and 1 blocks over two slots), and layer by layer.
PATHS = {
    "single_stage": dict(blocks=12, chunk=32, h=4, per_layer=False, n=(1, 7)),
    "block_stages": dict(blocks=100, chunk=64, h=8, per_layer=False, n=(90, 98)),
    "per_layer": dict(blocks=12, chunk=32, h=4, per_layer=True, n=(1, 8)),
}


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_stream_hazards_under_random_delays(scb, oracle, seed, path):
    from speccache_b200.cache import KVRestorePipeline

    rng = random.Random(seed)
    geo = PATHS[path]
    layers, blocks, chunk, h, d = 6, geo["blocks"], geo["chunk"], geo["h"], 128
    with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, n_slots=2,
                           per_layer=geo["per_layer"]) as pipe:
        _fill(pipe, 10 + seed)
        jobs = []
        for _ in range(4):  # restores that reuse the slots and the shift metadata
            ids = rng.sample(range(blocks - 2), rng.randint(*geo["n"]))
            dps = [rng.randint(-5000, 5000) for _ in ids]
            k_out = torch.empty((layers, len(ids) * chunk, h, d), dtype=torch.float16, device=DEV)
            v_out = torch.empty_like(k_out)
            torch.cuda._sleep(rng.randint(0, 50) * CYCLES_PER_MS // 10)
            pipe.restore(ids, dps, list(k_out), list(v_out))
            time.sleep(rng.random() * 0.005)
            jobs.append((ids, dps, k_out, v_out))
        # the slabs as the restores read them (the offloads below overwrite other blocks)
        snapshot = [t.clone() for t in (pipe.k_quant, pipe.k_scale, pipe.v_quant, pipe.v_scale)]
        # offloads that reuse both offload slots, each after a delay on the compute stream,
        # then a restore of the offloaded blocks, ordered after them on the transfer stream
        g = torch.Generator().manual_seed(seed)
        off_ids = [blocks - 2, blocks - 1]
        fresh = []
        for layer in range(layers):
            k = torch.randn((len(off_ids) * chunk, h, d), generator=g).half()
            v = torch.randn((len(off_ids) * chunk, h, d), generator=g).half()
            torch.cuda._sleep(rng.randint(0, 20) * CYCLES_PER_MS // 10)
            pipe.offload(layer, off_ids, k.to(DEV), v.to(DEV))
            fresh.append((k, v))
        k_back = torch.empty((layers, len(off_ids) * chunk, h, d), dtype=torch.float16, device=DEV)
        v_back = torch.empty_like(k_back)
        pipe.restore(off_ids, [0, 0], list(k_back), list(v_back))
        pipe.synchronize(timeout=60.0)
        assert pipe.status() == 0
        kq_s, ks_s, vq_s, vs_s = snapshot
        for ids, dps, k_out, v_out in jobs:
            for layer in range(layers):
                kr, vr = oracle.restore_blocks(kq_s[layer], ks_s[layer], vq_s[layer], vs_s[layer],
                                               ids, dps, 10000.0, torch.float16)
                torch.testing.assert_close(k_out[layer].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)
                assert bits_equal(v_out[layer].cpu(), vr)
        for layer, (k, v) in enumerate(fresh):
            kq, ks = oracle.quantize_kv_int8(k)
            vq, vs = oracle.quantize_kv_int8(v)
            assert bits_equal(v_back[layer].cpu(), oracle.dequant_value(vq, vs))
            c, s = oracle.compute_rope_cos_sin_delta(0, d)
            assert bits_equal(k_back[layer].cpu(), oracle.dequant_rope_shift(kq, ks, c, s))
