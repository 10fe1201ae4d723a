"""The C-ABI library loads here (no GPU) and exports what include/mpo_b200.h declares."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from mps_pointops import _native as N

HEADER = ROOT / "include" / "mpo_b200.h"


def declared() -> set[str]:
    return set(re.findall(r"^MPO_API\s+[\w\s\*]+?\b(mpo_\w+)\(", HEADER.read_text(), flags=re.M))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    names = declared()
    assert len(names) >= 16
    for name in names:
        assert hasattr(lib, name), name
    assert names == set(N.SIGNATURES), "ctypes signatures must mirror the header"


def test_abi_version_and_error_channel():
    lib = N.lib()
    assert lib.mpo_abi_version() == N.ABI_VERSION == 9
    # Argument validation happens before any CUDA call, so it runs without a GPU.
    st = lib.mpo_knn(None, None, 1, 1, 1000, 3, 300, None, None, None, None, 0, None)
    assert st == 1
    assert "at most 256" in N.last_error()
    # The tensor-core feature path needs a workspace; D == 3 needs none.
    assert lib.mpo_knn_workspace_bytes(2, 4096, 4096, 64, 20) > 2 * 4096 * 64 * 8
    assert lib.mpo_knn_workspace_bytes(2, 4096, 4096, 3, 20) == 0
    assert lib.mpo_knn_workspace_bytes(2, 4096, 1000, 64, 20) == 0
    st = lib.mpo_fps(None, 1, 10, 4, 12, 0, 0, 0, None, None, None, 0, None)
    assert st == 1 and "start_idx" in N.last_error()
    st = lib.mpo_fps(None, 1, 10, 4, 0, 0, 0, 7, None, None, None, 0, None)
    assert st == 1 and "strategy" in N.last_error()


def test_workspace_queries():
    lib = N.lib()
    assert lib.mpo_fps_workspace_bytes(8, 4096, 1024, 0) == 0
    assert lib.mpo_fps_workspace_bytes(1, 1 << 20, 65536, 0) > 0
    assert lib.mpo_fps_workspace_bytes(3, 100, 10, 2) >= 3 * 32
    assert lib.mpo_flat_fps_workspace_bytes(5, 8192) == 0
    assert lib.mpo_flat_fps_workspace_bytes(5, 20000) > 0


def test_flat_entry_points_validate_before_device_work():
    lib = N.lib()
    st = lib.mpo_flat_knn(None, None, None, None, 1, 10, 10, 3, 300, 10, None, None, None)
    assert st == 1 and "k must be in [0, 256]" in N.last_error()
    st = lib.mpo_flat_knn(None, None, None, None, 1, 10, 10, 3, 4, 10, None, None, None)
    assert st == 1 and "status" in N.last_error()
    st = lib.mpo_flat_radius(None, None, None, None, 1, 10, -1, 0.25, 4, 0, None, None, None)
    assert st == 1 and "negative size" in N.last_error()
    st = lib.mpo_flat_fps(None, None, None, None, 2, 10, 4, 5, None, None, None, 0, None)
    assert st == 1 and "status" in N.last_error()


def test_no_oracle_in_product_package():
    pkg = ROOT / "mps-pointops_b200"
    for path in pkg.rglob("*.py"):
        text = path.read_text()
        assert "oracle" not in text.replace("# ", ""), path
    for path in (pkg / "csrc").glob("*"):
        assert "oracle" not in path.read_text(), path


def test_peer_allreduce_validates_before_device_work():
    lib = N.lib()
    fake = ctypes.c_void_p(0x1000)
    slots = (ctypes.c_void_p * 2)(0x2000, 0x3000)
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, fake, slots, 2, 0, 0, 10, fake, None)
    assert st == 1 and "seq must not be 0" in N.last_error()
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, fake, slots, 33, 0, 1, 10, fake, None)
    assert st == 1 and "world must be in [1, 32]" in N.last_error()
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, fake, slots, 2, 2, 1, 10, fake, None)
    assert st == 1 and "rank must be in [0, world)" in N.last_error()
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, fake, slots, 2, 0, 1, 0, fake, None)
    assert st == 1 and "timeout_ns" in N.last_error()
    bad = (ctypes.c_void_p * 2)(0x2000, 0x3004)
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, fake, bad, 2, 0, 1, 10, fake, None)
    assert st == 1 and "slots[1]" in N.last_error()
    st = lib.mpo_allreduce_sum_f32_p2p(fake, 1.0, None, slots, 2, 0, 1, 10, fake, None)
    assert st == 1 and "must not be NULL" in N.last_error()
