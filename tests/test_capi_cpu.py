"""The C-ABI library on a machine without a GPU: it loads, exports every entry point that
include/cab_capi.h declares, and rejects bad arguments before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest

from cab_attention import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "cab_capi.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"CAB_API\s+[\w\s\*]+?\b(cab_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent /
                           "bridge-aware-kv-cache-eviction-for-efficient-long-context-transformers_b200"))
    import cab_build
    cab_build.build()
    return _lib.lib()


def test_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes binding out of sync with the header"


def test_version_and_error_string(lib):
    assert lib.cab_get_version() == 1
    rc = lib.cab_topk_blocks(None, None, None, None, 1, 4, 1, 1, 1, 0, None)
    assert rc == 1
    assert b"NULL" in lib.cab_last_error_string()


def test_argument_checks_without_gpu(lib):
    fake = ctypes.c_void_p(16)
    # k outside [1, M]
    assert lib.cab_topk_blocks(fake, fake, fake, None, 1, 8, 9, 1, 1, 0, None) == 1
    # unknown dtype
    s = _lib._i64_3(1, 1, 1)
    assert lib.cab_coarsen_maxl2(fake, None, fake, None, None, None, 1, 1, 0, 64, 64, 64, s, None,
                                 7, None) == 2
    # workspace too small
    n = _lib._c_size(0)
    assert lib.cab_frc_workspace_size(1, 2, 100, 64, 2, 0, ctypes.byref(n)) == 0 and n.value > 0
    assert lib.cab_frc(fake, fake, fake, None, None, 1, 2, 2, 100, 64, 2, 1.0, 0.5, 0, 0, 0,
                       fake, 16, None) == 5
    # Hq not a multiple of Hkv
    assert lib.cab_frc(fake, fake, fake, None, None, 1, 3, 2, 100, 64, 2, 1.0, 0.5, 0, 0, 0,
                       fake, n.value, None) == 1
    # host prefill: NULL input, keep outside [1, M], host memory that is not page-locked
    args = (1, 2, 2, 256, 64, 64)
    assert lib.cab_prefill_host(None, fake, fake, fake, None, None, *args, 1, 1.0, 0.5, 0, 0, 0,
                                1, 1, 0, 0.125, 2, fake, 1 << 30, None) == 1
    assert lib.cab_prefill_host(fake, fake, fake, fake, None, None, *args, 5, 1.0, 0.5, 0, 0, 0,
                                1, 1, 0, 0.125, 2, fake, 1 << 30, None) == 1
    buf = ctypes.create_string_buffer(2 * 256 * 64 * 2)
    hb = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.cab_prefill_host(hb, hb, hb, hb, None, None, *args, 1, 1.0, 0.5, 0, 0, 0,
                                1, 1, 0, 0.125, 2, fake, 1 << 30, None) == 1
    assert b"page-locked" in lib.cab_last_error_string()


def test_workspace_queries(lib):
    n = _lib._c_size(0)
    assert lib.cab_sparse_attn_workspace_size(2, 8, 128000, 128, 64, 100, 2, ctypes.byref(n)) == 0
    assert n.value >= 2 * 8 * 1000 * (2 * 100 + 2) * 4
    assert lib.cab_sparse_attn_workspace_size(1, 8, 4096, 64, 64, 6, 0, ctypes.byref(n)) == 0
    assert n.value == 0  # fp32 runs the CUDA-core kernel, which needs no scratch
    # host prefill: two slots of one (b, KV head) unit, independent of B and Hkv
    one = _lib._c_size(0)
    assert lib.cab_prefill_host_workspace_size(1, 8, 8, 128000, 128, 64, 100, 2, 0,
                                               ctypes.byref(one)) == 0
    assert lib.cab_prefill_host_workspace_size(2, 8, 8, 128000, 128, 64, 100, 2, 0,
                                               ctypes.byref(n)) == 0
    assert n.value == one.value and n.value >= 2 * (4 * 128000 * 128 * 2 + 2000 * 2000 * 4)


def test_ops_refuse_cpu_tensors():
    import torch
    from cab_attention.kernels import coarsen_qk_max_l2
    q = torch.randn(1, 1, 64, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        coarsen_qk_max_l2(q, q)


def test_roofline_formulas_match_the_documented_sizes():
    from cab_attention import roofline as rl
    # north_star: 1065 MB coarsening, 16.4 + 256 GFLOP FRC, 269 MB top-k, 6.71 TFLOP attention
    assert abs(rl.coarsen_bytes(2, 8, 8, 128000, 128) / 1e6 - 1065) < 1
    assert abs(rl.frc_flops(2, 8, 2000, 128) / 1e9 - 272.4) < 0.1
    assert abs(rl.topk_bytes(2, 8, 2000, 100) / 1e6 - 268.9) < 0.1
    assert abs(rl.sparse_attention_flops(3_200_000, 64, 128) / 1e12 - 6.71) < 0.01
    achieved, frac = rl.fraction(1065e6, 0.2, 6456.5, "GB/s")
    assert abs(achieved - 5325) < 1 and 0.8 < frac < 0.85


def test_clock_sampler_reports_only_the_timed_window():
    """bench.py's clock record: samples outside [mark_start, mark_end] (the idle lead-in
    and tail) are dropped, NVML reason bits map to their names."""
    import sys
    import time
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import bench
    s = bench.ClockSampler(0)
    s.mode, s.max_mhz = "nvml", 1965.0
    now = time.monotonic()
    s.samples = [(now - 1.0, 1965.0, 0, 100.0), (now + 0.1, 1500.0, 0x4, 990.0),
                 (now + 0.2, 1520.0, 0x4 | 0x8, 995.0), (now + 5.0, 1965.0, 0, 120.0)]
    s.t0, s.t1 = now, now + 1.0
    c = s.stop()
    assert c["samples"] == 2 and c["sm_mhz"] == 1510.0 and c["sm_max_mhz"] == 1965.0
    assert c["reasons"] == ["hw_slowdown", "sw_power_cap"]
