"""The reference engine itself, built from its own sources (integration/):
model_load + model_forward on a one-layer GGUF (tests/gguf_writer.py:
attention weights zero, norm weights one, identity output head, so the logits
are x + MoE(rmsnorm(x))).

* CPU: the unmodified engine (its CPU backend) against x + the oracle's MoE
  layer (renorm 0, ungated shared expert, interleaved slices: the engine as
  shipped) — the cross-check of the oracle's restatement of
  engine/src/model.c:992-1143 against the real model_forward.
* GPU: the engine linked against libornith_cuda.so with the routed-expert
  block on gpu_moe_forward (patch_model_moe.py) against the unmodified CPU
  engine on the same file, per token within 1e-3 relative."""
import os
import subprocess

import numpy as np
import pytest

from gguf_writer import engine_model_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT = os.path.join(ROOT, "integration", "_out")


def run_engine(name, gguf, token, tmp_path):
    exe = os.path.join(OUT, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (needs the reference tree at build time)")
    out = str(tmp_path / f"{name}_{token}.bin")
    r = subprocess.run([exe, gguf, str(token), out], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.fromfile(out, np.float32)


@pytest.fixture(scope="module")
def model_file(oracle, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("engine") / "one_layer.gguf")
    w, emb = engine_model_gguf(path, oracle)
    return path, w, emb


def test_reference_engine_matches_oracle_layer(oracle, model_file, tmp_path):
    path, w, emb = model_file
    cfg = dict(d_model=256, hidden=256, n_experts=8, top_k=2, layout=1, routing=0, renorm=0, shared_gate=0)
    for token in (0, 3, 101):
        got = run_engine("engine_cpu", path, token, tmp_path)
        x = emb[:, token].astype(np.float32)
        xn = (x / np.sqrt((x * x).mean(dtype=np.float32) + np.float32(1e-6))).astype(np.float32)
        want, _, _ = oracle.moe_forward(cfg, w, xn[None])
        ref = x + want[0]
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max(), token


@pytest.mark.gpu
def test_engine_on_cuda_backend_matches_cpu_engine(cuda, model_file, tmp_path):
    path, _, _ = model_file
    for token in (0, 3, 101, 255):
        cpu = run_engine("engine_cpu", path, token, tmp_path)
        gpu = run_engine("engine_cuda", path, token, tmp_path)
        err = np.abs(gpu - cpu).max() / np.abs(cpu).max()
        assert err <= 1e-3, (token, err)
