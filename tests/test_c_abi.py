"""The C ABI used from C alone: tests/c_abi_consumer.c, a C11 program with no Python or torch
in its process, built with gcc against include/speccache_b200.h and the in-tree library.

* CPU: the header and the consumer compile as strict C11 and link against the library's
  exported symbols.
* GPU: the consumer quantizes seeded fp32 K/V, restores them with an in-library shift table
  and writes everything to a file; codes and scales must equal the oracle's bit for bit, V
  too, and K must lie within the reference tolerance (rtol = atol = 1e-2).  It then restores 9
  scattered blocks of a 3-layer pinned-host pipeline whose slabs it filled from C; every layer
  is checked against the oracle the same way, and the plan it read must be 3 launches (two
  block stages and the scale gather) and 7 copy commands.
"""

from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from conftest import REPO, bits_equal

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
SRC = os.path.join(REPO, "tests", "c_abi_consumer.c")
LIB_DIR = os.path.join(REPO, "intelligent-bell_b200")

pytestmark = pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")


def _build(scb, out_dir: str) -> str:
    scb._lib.load()  # the library exists (build() has run)
    exe = os.path.join(out_dir, "c_abi_consumer")
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-pedantic",
           f"-I{os.path.join(REPO, 'include')}", f"-I{os.path.join(CUDA_HOME, 'include')}", SRC,
           "-o", exe, f"-L{LIB_DIR}", "-lspeccache_b200", f"-Wl,-rpath,{LIB_DIR}",
           f"-L{os.path.join(CUDA_HOME, 'lib64')}", "-lcudart",
           f"-Wl,-rpath,{os.path.join(CUDA_HOME, 'lib64')}"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr
    return exe


def test_consumer_compiles_as_c11_and_links(scb, tmp_path):
    assert os.path.isfile(_build(scb, str(tmp_path)))


def _read(path):
    with open(path, "rb") as f:
        raw = f.read()
    t, h, d = np.frombuffer(raw, np.int32, 3, 0)
    dp, theta = np.frombuffer(raw, np.float64, 2, 12)
    n, rows, off = int(t) * int(h) * int(d), int(t) * int(h), 28
    out = {}
    for name, dtype, count in (("xk", np.float32, n), ("xv", np.float32, n), ("kq", np.int8, n),
                               ("vq", np.int8, n), ("ks", np.int16, rows), ("vs", np.int16, rows),
                               ("ko", np.int16, n), ("vo", np.int16, n)):
        a = np.frombuffer(raw, dtype, count, off).copy()
        off += a.nbytes
        out[name] = torch.from_numpy(a)
    # the pipeline section
    pl, pb, pc, ph, pd, pn, launches, copies = (int(x) for x in np.frombuffer(raw, np.int32, 8, off))
    off += 32
    pipe = {"geo": (pl, pb, pc, ph, pd), "launches": launches, "copies": copies}
    slab, slab_s, outs = pl * pb * pc * ph * pd, pl * pb * pc * ph, pl * pn * pc * ph * pd
    for name, dtype, count in (("ids", np.int32, pn), ("shifts", np.int32, pn),
                               ("kq", np.int8, slab), ("vq", np.int8, slab),
                               ("ks", np.int16, slab_s), ("vs", np.int16, slab_s),
                               ("ko", np.int16, outs), ("vo", np.int16, outs)):
        a = np.frombuffer(raw, dtype, count, off).copy()
        off += a.nbytes
        pipe[name] = torch.from_numpy(a)
    assert off == len(raw)
    for k in ("kq", "vq"):
        pipe[k] = pipe[k].view(pl, pb, pc, ph, pd)
    for k in ("ks", "vs"):
        pipe[k] = pipe[k].view(torch.float16).view(pl, pb, pc, ph, 1)
    for k in ("ko", "vo"):
        pipe[k] = pipe[k].view(torch.float16).view(pl, pn * pc, ph, pd)
    out["pipeline"] = pipe
    shape, sshape = (int(t), int(h), int(d)), (int(t), int(h), 1)
    for k in ("xk", "xv", "kq", "vq", "ko", "vo"):
        out[k] = out[k].view(shape)
    for k in ("ks", "vs"):
        out[k] = out[k].view(sshape)
    for k in ("ks", "vs", "ko", "vo"):
        out[k] = out[k].view(torch.float16)
    return out, float(dp), float(theta)


@pytest.mark.gpu
@pytest.mark.parametrize("geo", [(1, 1, 64, -384, 1e4), (300, 8, 128, 4095, 5e5),
                                 (77, 3, 96, -70000, 1e6)])
def test_consumer_restores_like_the_oracle(scb, oracle, tmp_path, geo):
    exe = _build(scb, str(tmp_path))
    t, h, d, dp, theta = geo
    out_file = os.path.join(str(tmp_path), "out.bin")
    proc = subprocess.run([exe, out_file, str(t), str(h), str(d), str(dp), str(theta)],
                          capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "rejected call: rc=" in proc.stdout
    r, dp_f, theta_f = _read(out_file)
    assert (dp_f, theta_f) == (float(dp), float(theta))
    for x, q, s in (("xk", "kq", "ks"), ("xv", "vq", "vs")):
        q_ref, s_ref = oracle.quantize_kv_int8(r[x])
        assert torch.equal(r[q], q_ref)
        assert bits_equal(r[s], s_ref)
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, theta)
    k_ref = oracle.dequant_rope_shift(r["kq"], r["ks"], cos, sin)
    torch.testing.assert_close(r["ko"], k_ref, rtol=1e-2, atol=1e-2)
    assert bits_equal(r["vo"], oracle.dequant_value(r["vq"], r["vs"]))
    pipe = r["pipeline"]
    assert (pipe["launches"], pipe["copies"]) == (3, 7)
    ids, shifts = pipe["ids"].tolist(), pipe["shifts"].tolist()
    for layer in range(pipe["geo"][0]):
        kr, vr = oracle.restore_blocks(pipe["kq"][layer], pipe["ks"][layer], pipe["vq"][layer],
                                       pipe["vs"][layer], ids, shifts, theta, torch.float16)
        assert bits_equal(pipe["vo"][layer], vr), layer
        torch.testing.assert_close(pipe["ko"][layer], kr, rtol=1e-2, atol=1e-2)
