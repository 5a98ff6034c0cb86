"""CPU: the C ABI library loads, exports every declared symbol, and rejects bad
arguments before touching the device; the Python surfaces mirror the
reference's names and exceptions.  No kernel is launched here."""
from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from pathtile_b200 import _lib, ops, runtime, warp_tiled

HEADER = ROOT / "include" / "pathtile_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pt_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_api():
    names = declared_functions()
    for n in ("pt_fwd", "pt_dx", "pt_dk", "pt_dk_workspace_bytes", "pt_config"):
        assert n in names


def test_library_exports_every_declared_symbol(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), name
        assert name in _lib.SIGNATURES, f"{name} lacks a ctypes signature"


def test_version_and_status_strings(native_lib):
    assert native_lib.pt_version() >= 100
    for st in (0, -2, -3, -4, -5, -6, -7, -8):
        assert _lib.status_string(st)
    assert "L <= 48" in _lib.status_string(_lib.PT_ERR_UNSUPPORTED)


FAKE = ctypes.c_void_p(0x10000)  # aligned, never dereferenced: checks fail before any CUDA call
MISALIGNED = ctypes.c_void_p(0x10004)
NULL = ctypes.c_void_p(0)


@pytest.mark.parametrize(
    "args,status",
    [
        ((NULL, FAKE, FAKE, 2, 4, 16, 8), _lib.PT_ERR_ARGS),
        ((FAKE, FAKE, FAKE, 2, 0, 16, 8), _lib.PT_ERR_ARGS),
        ((FAKE, FAKE, FAKE, -1, 4, 16, 8), _lib.PT_ERR_ARGS),
        ((FAKE, FAKE, FAKE, 2, 4, 49, 8), _lib.PT_ERR_UNSUPPORTED),
        ((FAKE, FAKE, FAKE, 2, 4, 16, 49), _lib.PT_ERR_UNSUPPORTED),
        ((FAKE, FAKE, MISALIGNED, 2, 4, 16, 8), _lib.PT_ERR_ALIGN),
        ((FAKE, FAKE, FAKE, 0, 4, 16, 8), _lib.PT_OK),  # empty batch: nothing to do
    ],
)
def test_fwd_dx_argument_checks(native_lib, args, status):
    assert native_lib.pt_fwd(*args, NULL) == status
    assert native_lib.pt_dx(*args, NULL) == status


def test_dk_argument_checks(native_lib):
    assert native_lib.pt_dk(FAKE, FAKE, FAKE, 2, 4, 16, 8, 7, NULL, 0, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_dk(FAKE, NULL, FAKE, 2, 4, 16, 8, 0, NULL, 0, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_dk(FAKE, FAKE, FAKE, 2, 4, 16, 50, 0, NULL, 0, NULL) == _lib.PT_ERR_UNSUPPORTED
    assert native_lib.pt_dk(MISALIGNED, FAKE, FAKE, 2, 4, 16, 8, 0, NULL, 0, NULL) == _lib.PT_ERR_ALIGN
    assert native_lib.pt_dk(FAKE, FAKE, FAKE, 0, 4, 16, 8, 0, NULL, 0, NULL) == _lib.PT_OK
    assert native_lib.pt_dk_workspace_bytes(0, 4, 16, 8) == 0
    assert native_lib.pt_dk_workspace_bytes(2, 4, 49, 8) == 0


def test_set_config_validation(native_lib):
    assert native_lib.pt_set_config(0, 100, 3, 2, 1) == _lib.PT_ERR_ARGS
    assert native_lib.pt_set_config(0, 128, 5, 2, 1) == _lib.PT_ERR_ARGS
    assert native_lib.pt_set_config(0, 128, 3, 9, 1) == _lib.PT_ERR_ARGS
    assert native_lib.pt_set_config(3, 128, 3, 2, 1) == _lib.PT_ERR_ARGS
    assert native_lib.pt_set_config(0, 128, 3, 2, 3) == _lib.PT_ERR_ARGS
    assert native_lib.pt_set_config(0, 64, 2, 1, 2) == _lib.PT_OK
    cfg = ops.config("fwd", 16384, 128, 48, 48)
    assert cfg["rows_per_tile"] == 64 and cfg["stages"] == 2 and cfg["threads_per_row"] == 2
    assert native_lib.pt_set_config(0, 0, 0, 0, 0) == _lib.PT_OK


def test_per_call_options_validation_and_effect(native_lib):
    o = _lib.LaunchOpts.frozen()
    o.rows_per_tile[0], o.stages[0], o.ctas_per_sm[0], o.threads_per_row[0] = 64, 2, 1, 2
    po = ctypes.cast(ctypes.pointer(o), ctypes.c_void_p)
    # Per-call options change that call's plan only; the process-wide choice stays frozen.
    assert ops.config("fwd", 16384, 128, 48, 48, opts=o)["rows_per_tile"] == 64
    assert ops.config("fwd", 16384, 128, 48, 48)["rows_per_tile"] == 128
    assert native_lib.pt_fwd_ex(FAKE, FAKE, FAKE, 0, 4, 16, 8, po, NULL) == _lib.PT_OK
    bad = _lib.LaunchOpts.frozen()
    bad.rows_per_tile[2], bad.stages[2], bad.ctas_per_sm[2], bad.threads_per_row[2] = 100, 3, 2, 1
    pb = ctypes.cast(ctypes.pointer(bad), ctypes.c_void_p)
    assert native_lib.pt_fwd_ex(FAKE, FAKE, FAKE, 2, 4, 16, 8, pb, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_dk_ex(FAKE, FAKE, FAKE, 2, 4, 16, 8, 1, NULL, 0, pb, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_dk_workspace_bytes_ex(2, 4, 16, 8, pb) == 0
    eng = _lib.LaunchOpts.frozen()
    eng.engine[1] = 7
    pe = ctypes.cast(ctypes.pointer(eng), ctypes.c_void_p)
    assert native_lib.pt_dx_ex(FAKE, FAKE, FAKE, 2, 4, 16, 8, pe, NULL) == _lib.PT_ERR_ARGS
    out = (ctypes.c_int * 7)()
    assert native_lib.pt_config_ex(0, 16, 4, 16, 8, out, 7, pe) == _lib.PT_ERR_ARGS
    bk = _lib.LaunchOpts.frozen()
    bk.bwd_kernel = 4
    pk = ctypes.cast(ctypes.pointer(bk), ctypes.c_void_p)
    assert native_lib.pt_dx_dk_ex(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 4, 16, 8, 1, NULL, 0, pk, NULL) == _lib.PT_ERR_ARGS
    bk.bwd_kernel, bk.helper_channels = _lib.PT_BWD_SEPARATE, -2
    assert native_lib.pt_dx_dk_ex(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 4, 16, 8, 1, NULL, 0, pk, NULL) == _lib.PT_ERR_ARGS


def test_runtime_launch_options_map_reference_arguments():
    o = runtime.launch_options(warps_per_block=2, bwdk_block=256, stages=4, ctas_per_sm=1)
    assert list(o.rows_per_tile) == [64, 64, 256]
    assert list(o.stages) == [4, 4, 4] and list(o.ctas_per_sm) == [1, 1, 1]
    assert list(o.engine) == [-1, -1, -1]
    f = runtime.launch_options()
    assert list(f.rows_per_tile) == [0, 0, 0]  # all frozen


def test_peer_exchange_argument_checks(native_lib):
    assert native_lib.pt_peer_buffer_bytes(0, 128, 48) == 0
    assert native_lib.pt_peer_buffer_bytes(9, 128, 48) == 0
    assert native_lib.pt_peer_buffer_bytes(2, 128, 48) == 2 * 2 * 128 * 48 * 4 + 2 * 2 * 128 * 4
    grp = _lib.PeerGroup(0, 2, (ctypes.c_void_p * _lib.PT_MAX_PEERS)(0x10000, 0x20000), 0)
    pg = ctypes.cast(ctypes.pointer(grp), ctypes.c_void_p)
    # epoch 0 and a missing group are rejected before any CUDA call
    assert native_lib.pt_dx_dk_allreduce(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 4, 16, 8, NULL, 0, pg, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_dx_dk_allreduce(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 4, 16, 8, NULL, 0, NULL, NULL) == _lib.PT_ERR_ARGS
    grp.epoch, grp.world = 1, 1
    assert native_lib.pt_allreduce_peer(FAKE, 4, 8, pg, NULL) == _lib.PT_ERR_ARGS
    grp.world, grp.rank = 2, 2
    assert native_lib.pt_allreduce_peer(FAKE, 4, 8, pg, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_peer_alloc(0, ctypes.byref(ctypes.c_void_p())) == _lib.PT_ERR_ARGS


def test_wait_selftest_argument_checks(native_lib):
    assert native_lib.pt_selftest_wait_timeout(0, FAKE, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_selftest_wait_timeout(2_000_000_000, FAKE, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_selftest_wait_timeout(1000, NULL, NULL) == _lib.PT_ERR_ARGS
    assert native_lib.pt_selftest_wait_timeout(1000, MISALIGNED, NULL) == _lib.PT_ERR_ALIGN


def test_frozen_config_and_specialisation_flags(native_lib):
    cfg = ops.config("fwd", 16384, 128, 48, 48)
    assert cfg["specialised"] == 1
    assert ops.config("bwd_weight", 4096, 64, 37, 13)["specialised"] == 1  # H*L % 4 == 0: bulk path
    assert ops.config("bwd_weight", 4096, 63, 37, 13)["specialised"] == 0  # misaligned rows: generic
    assert ops.config("fwd", 8, 8, 23, 11)["specialised"] == 0  # not in the table: generic


def test_python_checks_mirror_reference_exceptions():
    x = torch.zeros(2, 4, 16)
    k = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="CUDA"):
        ops.check_shapes(x, k)
    with pytest.raises(ValueError, match="CUDA"):
        warp_tiled.depthwise_conv_shared(x, k)
    with pytest.raises(ValueError, match="CUDA"):
        ops.dk(x, x, k)


def test_legacy_surface_names():
    for name in warp_tiled.__all__:
        assert hasattr(warp_tiled, name)
    assert warp_tiled.THREADS_PER_BLOCK == 512
    assert warp_tiled.shared_memory_bytes(48) == 16 * (32 + 47) * 4
    assert warp_tiled.bwd_kernel_shared_memory_bytes(48) == 2 * 64 * 48 * 4
    warp_tiled.FWD_TIMES.append(1.0)
    warp_tiled.reset_timing_collectors()
    assert warp_tiled.FWD_TIMES == [] and warp_tiled.BWD_K_TIMES == []


def test_runtime_surface_names_and_helpers():
    assert runtime.AmpereWarpRuntime is runtime.B200WarpRuntime
    assert runtime.DepthConvAmpere is runtime.DepthConvB200
    assert runtime.minimum_algorithmic_bytes(16384, 128, 48, 48) == 805_330_944
    assert runtime.in_range_pairs(48, 48) == 1728
    assert runtime.algorithmic_flops(16384, 128, 48, 48) == 7_247_757_312
    with pytest.raises(RuntimeError, match="installed"):
        runtime._RUNTIME = None
        runtime.get_runtime()


@pytest.mark.parametrize("L,K", [(1, 1), (1, 48), (48, 1), (5, 48), (37, 13), (48, 3), (33, 33), (16, 4)])
def test_in_range_pairs_brute_force(L, K):
    pad = K // 2
    brute = sum(1 for t in range(L) for j in range(K) if 0 <= t + j - pad < L)
    assert runtime.in_range_pairs(L, K) == brute


def test_occupancy_estimate_b200():
    prof = runtime.GPU_PROFILES[(10, 0)]
    est = runtime.estimate_gpu_occupancy(128, 117, 80 * 1024, prof)
    assert est["resident_blocks_per_sm_est"] == 2  # shared memory bound
    assert est["limiting_resources_est"] == "shared_memory"


def test_kernel_event_collector_disabled_runs_launch():
    c = runtime.KernelEventCollector()
    hits = []
    c.launch("fwd", lambda: hits.append(1))
    assert hits == [1] and c.resolve_rows(synchronize=False) == []


def test_summarize_kernel_times():
    rows = [{"phase": "fwd", "runtime_ms": v} for v in (1.0, 2.0, 3.0)]
    s = runtime.summarize_kernel_times(rows)[0]
    assert s["runs"] == 3 and s["mean_ms"] == 2.0 and s["median_ms"] == 2.0


def test_product_never_imports_the_oracle():
    pkg = ROOT / "pathtile_b200"
    for py in pkg.rglob("*.py"):
        text = py.read_text()
        assert "import oracle" not in text and "from oracle" not in text, py
