"""The native C bridge (include/cutechronos_bridge.h): the reference's
init / predict_median / destroy entry points (cutechronos_bridge.c:96-406),
served by the engine without Python.

CPU tests: the symbols are exported and every argument error that is found
before the device is touched comes back as -1 with the reference's message.
GPU tests: the bridge's median equals CuteChronos2Pipeline.predict_quantiles'
median bit for bit (same checkpoint, same kernels), matches the CPU oracle,
and a gcc-built C host gets the same numbers."""

from __future__ import annotations

import math
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import small_config, write_checkpoint
from cutechronos_b200 import _native as nat
from cutechronos_b200.foreign import BridgeError, NativeBridge
from cutechronos_b200.model import CuteChronos2Model
from cutechronos_b200.workloads import seeded_init_

ROOT = Path(__file__).resolve().parents[1]
BRIDGE_FUNCS = ("cutechronos_init_pipeline", "cutechronos_predict_median", "cutechronos_destroy_pipeline")


@pytest.fixture(scope="module")
def bridge():
    if not nat.LIB_PATH.exists():
        from cutechronos_b200 import build
        build.build()
    return NativeBridge(nat.load())


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    write_checkpoint(seeded_init_(CuteChronos2Model(small_config()), seed=5), d)
    return d


def test_header_declares_and_library_exports_bridge(bridge):
    text = (ROOT / "include" / "cutechronos_bridge.h").read_text()
    declared = set(re.findall(r"CC2_BRIDGE_API\s+int\s+(cutechronos_\w+)\s*\(", text))
    assert declared == set(BRIDGE_FUNCS)
    for n in BRIDGE_FUNCS:
        assert hasattr(bridge._lib, n)


@pytest.mark.parametrize("kw, msg", [
    (dict(backend="original"), "Unsupported backend 'original'"),
    (dict(dtype_name="float64"), "Unsupported dtype 'float64'"),
    (dict(device="cpu"), "unsupported device 'cpu'"),
])
def test_init_argument_errors(bridge, ckpt, kw, msg):
    with pytest.raises(BridgeError, match=re.escape(msg)):
        bridge.init_pipeline(str(ckpt), **kw)


def test_init_checkpoint_errors(bridge, tmp_path, ckpt):
    with pytest.raises(BridgeError, match="model_id is required"):
        bridge.init_pipeline("")
    with pytest.raises(BridgeError, match="No model weights found"):
        bridge.init_pipeline(str(tmp_path))
    # a truncated tensor section and a missing tensor are reported by name
    bad = tmp_path / "bad"
    bad.mkdir()
    (bad / "config.json").write_text((ckpt / "config.json").read_text())
    blob = (ckpt / "model.safetensors").read_bytes()
    (bad / "model.safetensors").write_bytes(blob[:len(blob) // 2])
    with pytest.raises(BridgeError, match="tensor .* has .* bytes|out of range"):
        bridge.init_pipeline(str(bad))
    from safetensors.torch import load_file, save_file
    sd = load_file(str(ckpt / "model.safetensors"))
    sd.pop("encoder.block.1.layer.2.mlp.wo.weight")
    save_file(sd, str(bad / "model.safetensors"))
    with pytest.raises(BridgeError, match="missing tensor encoder.block.1.layer.2.mlp.wo.weight"):
        bridge.init_pipeline(str(bad))
    (bad / "config.json").write_text('{"d_model": 128,')
    with pytest.raises(BridgeError, match="JSON parse error"):
        bridge.init_pipeline(str(bad))


def test_unknown_handle(bridge):
    with pytest.raises(BridgeError, match="unknown pipeline handle 12345"):
        bridge.predict_median(12345, [1.0, 2.0], 4)
    with pytest.raises(BridgeError, match="unknown pipeline handle 12345"):
        bridge.destroy_pipeline(12345)


# ---------------------------------------------------------------------------------------- GPU --
def _series(n, seed, nan_frac=0.0):
    g = torch.Generator().manual_seed(seed)
    x = 50 + 10 * torch.sin(torch.arange(n) / 7.0) + torch.randn(n, generator=g)
    if nan_frac:
        x[torch.rand(n, generator=g) < nan_frac] = float("nan")
    return x


def _pipeline_median(ckpt, dtype, ctx, H):
    from cutechronos_b200.pipeline import CuteChronos2Pipeline
    p = CuteChronos2Pipeline.from_pretrained(str(ckpt), device="cuda", dtype=dtype)
    q, _ = p.predict_quantiles(ctx, prediction_length=H, quantile_levels=[0.5])
    return q[0][0, :, 0]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name, dtype", [("bfloat16", torch.bfloat16), ("float32", torch.float32)])
@pytest.mark.parametrize("L, H, nan_frac", [(300, 24, 0.0), (700, 64, 0.02), (17, 5, 0.0)])
def test_bridge_equals_pipeline(bridge, ckpt, dtype_name, dtype, L, H, nan_frac):
    ctx = _series(L, seed=L + H, nan_frac=nan_frac)
    h = bridge.init_pipeline(str(ckpt), dtype_name=dtype_name)
    try:
        y, ms = bridge.predict_median(h, ctx.tolist(), H)
    finally:
        bridge.destroy_pipeline(h)
    ref = _pipeline_median(ckpt, dtype, ctx, H)
    assert len(y) == H and ms > 0
    assert torch.equal(torch.tensor(y), ref), (torch.tensor(y) - ref).abs().max()


@pytest.mark.gpu
def test_bridge_f32_vs_oracle(bridge, ckpt):
    from conftest import oracle_config
    from oracle import chronos2_oracle as orc
    from safetensors.torch import load_file
    ctx = _series(400, seed=11, nan_frac=0.01)
    H = 40
    h = bridge.init_pipeline(str(ckpt), dtype_name="float32")
    y, _ = bridge.predict_median(h, ctx.tolist(), H)
    bridge.destroy_pipeline(h)
    m = CuteChronos2Model(small_config())
    m.load_chronos2_weights(load_file(str(ckpt / "model.safetensors")))
    W = dict(m.named_parameters())
    ref = orc.forward(oracle_config(), W, ctx.view(1, -1), None, math.ceil(H / 16))
    mi = m.config.quantiles.index(0.5)
    assert (torch.tensor(y) - ref[0, mi, :H]).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-4


@pytest.mark.gpu
def test_bridge_graph_replay_and_shapes(bridge, ckpt):
    """compile_mode set: one CUDA graph per (L, N), replays equal the eager
    run, and switching shapes (which regrows the buffers) stays correct."""
    h_e = bridge.init_pipeline(str(ckpt))
    h_g = bridge.init_pipeline(str(ckpt), compile_mode="reduce-overhead")
    try:
        for L, H in [(256, 16), (256, 16), (1024, 128), (256, 16), (513, 33), (1024, 128)]:
            ctx = _series(L, seed=L).tolist()
            ye, _ = bridge.predict_median(h_e, ctx, H)
            yg, _ = bridge.predict_median(h_g, ctx, H)
            assert ye == yg
    finally:
        bridge.destroy_pipeline(h_e)
        bridge.destroy_pipeline(h_g)


@pytest.mark.gpu
def test_bridge_long_context_and_limits(bridge, ckpt):
    h = bridge.init_pipeline(str(ckpt))
    try:
        ctx = _series(900, seed=3)
        y_long, _ = bridge.predict_median(h, ctx.tolist(), 16)
        y_tail, _ = bridge.predict_median(h, ctx[-512:].tolist(), 16)  # context_length 512 keeps the tail
        assert y_long == y_tail
        with pytest.raises(BridgeError, match=r"prediction_length \(1025\) exceeds model_prediction_length \(1024\)"):
            bridge.predict_median(h, ctx.tolist(), 1025)
        with pytest.raises(BridgeError, match="forecast buffer too small"):
            bridge.predict_median(h, ctx.tolist(), 32, capacity=16)
        with pytest.raises(BridgeError, match="at least one value"):
            bridge.predict_median(h, [], 16)
        y_max, _ = bridge.predict_median(h, ctx.tolist(), 1024)
        assert len(y_max) == 1024 and np.isfinite(y_max).all()
    finally:
        bridge.destroy_pipeline(h)
    with pytest.raises(BridgeError, match="unknown pipeline handle"):
        bridge.predict_median(h, [1.0], 1)


@pytest.mark.gpu
def test_c_host_runner(bridge, ckpt, tmp_path):
    exe = tmp_path / "bridge_runner"
    lib_dir = nat.LIB_PATH.parent
    subprocess.run(["gcc", "-O2", "-std=c99", str(ROOT / "tests" / "bridge_runner.c"), "-I", str(ROOT / "include"),
                    "-L", str(lib_dir), "-lcc2_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    ctx = _series(333, seed=8, nan_frac=0.02)
    text = " ".join("nan" if math.isnan(v) else repr(v) for v in ctx.tolist())
    for dtype_name, mode in [("bfloat16", "-"), ("float32", "reduce-overhead")]:
        r = subprocess.run([str(exe), str(ckpt), dtype_name, mode, "20", "3"], input=text, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        lines = r.stdout.strip().splitlines()
        assert lines[-1].startswith("latency_ms ")
        y = torch.tensor([float(v) for v in lines[:-1]])
        h = bridge.init_pipeline(str(ckpt), dtype_name=dtype_name)
        ref, _ = bridge.predict_median(h, ctx.tolist(), 20)
        bridge.destroy_pipeline(h)
        assert torch.equal(y, torch.tensor(ref))
