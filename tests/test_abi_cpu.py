"""CPU-side checks of the C-ABI boundary: the library loads, exports every
entry point declared in include/torque_b200.h, the ctypes table matches the
header, and compute entry points fail loudly when no GPU is present."""

from __future__ import annotations

import ctypes
import re
import subprocess

import numpy as np
import pytest
import torch

from conftest import ROOT
from torque_mlx_b200 import _lib

HEADER = ROOT / "include" / "torque_b200.h"


def _declared() -> list[str]:
    text = HEADER.read_text()
    body = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tq_[a-z0-9_]+)\s*\(", body)))


@pytest.fixture(scope="module")
def built_lib():
    from torque_mlx_b200.build import build_library
    return build_library()


def test_header_declares_entry_points():
    names = _declared()
    assert "tq_decode" in names and "tq_append_kv" in names and len(names) >= 12


def test_ctypes_table_matches_header():
    assert sorted(_lib.SIGNATURES) == _declared()


def test_library_exports_every_declared_symbol(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(built_lib)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (tq_[a-z0-9_]+)$", out, flags=re.M))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing


def test_library_loads_and_reports_status(built_lib):
    lib = _lib.load(require_cuda=False)
    assert lib.tq_abi_version() == 1
    assert lib.tq_status_string(-2).decode().startswith("unsupported head dimension")


def test_host_side_argument_checks(built_lib):
    """Argument errors are caught on the host before any launch (no GPU needed)."""
    lib = _lib.load(require_cuda=False)
    assert lib.tq_rotate(None, 0, None, 4, 96, None, None, None) == _lib.TQ_E_HEAD_DIM
    assert lib.tq_quantize(None, None, 4, None, 5, None) == _lib.TQ_E_BITS
    assert lib.tq_pack(None, None, 0, 0, 3, None) == _lib.TQ_OK  # empty is a no-op
    size = ctypes.c_size_t()
    assert lib.tq_decode_workspace_size(4, 17, 128, 4, 100, 0, ctypes.byref(size)) == _lib.TQ_E_SHAPE
    assert lib.tq_decode_workspace_size(4, 4, 128, 4, 100, 0, ctypes.byref(size)) == _lib.TQ_OK
    assert size.value > 0
    assert lib.tq_decode(None, 0, None, None, None, None, 0, None, 1, 0, 0, 1, 1, 128, 4, None, None, 1.0,
                         None, None, 0, 0, None, 0, None) == _lib.TQ_E_ARG


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_compute_path_fails_loudly_without_gpu(built_lib):
    from torque_mlx_b200 import Codebook, TorqueConfig, TorqueKVCache, quantize
    cb = Codebook(bit_width=2, centroids=np.array([-1, -0.25, 0.25, 1], np.float32))
    with pytest.raises(RuntimeError, match="CUDA device"):
        quantize(np.zeros(4, np.float32), cb)
    with pytest.raises(RuntimeError, match="CUDA device"):
        TorqueKVCache(config=TorqueConfig(bit_width=4, head_dim=64))


def test_bench_arms_print_the_same_config():
    """bench.py's own arm and its --impl reference arm describe a workload with
    the same config dict (the driver compares them)."""
    import bench
    for name in ("config4", "config4_4bit", "config3", "longctx128"):
        wl = dict(bench.WORKLOADS[name])
        for world in (1, 2, 8):
            assert bench.config_dict(name, wl, world) == bench.config_dict(name, dict(wl), world)
            assert bench.config_dict(name, wl, world)["global_batch"] == wl["batch"] * world
