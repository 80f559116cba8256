"""bench.py reports each dominant kernel's DRAM traffic per launch from the ncu summaries
under profiles/ (`traffic_bytes_per_launch[<kernel>|<workload>|<units>]: <bytes>`).
Every kernel the bench can name as dominant must resolve to a recorded capture, and the
recorded traffic must stay within a plausible factor of the kernel's algorithmic bytes.
A profile that is renamed or edited would otherwise turn `roofline.traffic` into null
without any error."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
UNITS = 129_684  # sequence-steps of one op-level pass (404 x 321 = 1284 x 101)

# (kernel, bench workload tag, algorithmic bytes per sequence-step) for the kernels
# bench.py names: LinOSS P = 256; SISO C = 256, N = 16 (real / complex gamma); MIMO
# 8 heads x 32, state 128, rank 4 (bf16 input, 1872-column projection); the MIMO operator and
# the plain complex scan at 404 x 321, 8 heads x 16 modes, 32 channels per head.
CASES = [
    ("linoss_fwd_kernel", "linoss", 16 * 256),
    ("linoss_bwd_kernel", "linoss", 24 * 256),
    ("slru_fwd_kernel", "slru real", 4 * (3 * 256 + 2 * 16)),
    ("slru_fwd_real16_kernel", "slru real", 4 * (3 * 256 + 2 * 16)),
    ("slru_bwd_kernel", "slru real", 4 * (5 * 256 + 4 * 16)),
    ("slru_fwd_kernel", "slru complex", 4 * (4 * 256 + 4 * 16)),
    ("slru_bwd_kernel", "slru complex", 4 * (7 * 256 + 8 * 16)),
    ("mimo_layer_fwd_kernel", "mimo", 5280),
    ("mimo_layer_fwd_tc_kernel", "mimo", 5280),
    ("mimo_layer_bwd16_kernel", "mimo", 9536),
    ("mimo_layer_bwd_tc_kernel", "mimo", 9536),
    ("mimo_fwd_kernel", "ops", 24 * 128 + 8 * 256),
    ("mimo_bwd_kernel", "ops", 40 * 128 + 12 * 256),
    ("cscan_fwd_kernel", "ops_cscan", 24 * 128),
    ("cscan_bwd_kernel", "ops_cscan", 40 * 128),
    # per token row of the generator layer: C = 256, rank 4, P = 16
    ("step_proj_fwd_kernel", "surround_step", 8 * 256 + 4 * 4),
    ("step_proj_bwd_kernel", "surround_step", 8 * 256 + 8 * 4),
    ("linoss_readout_fwd_kernel", "surround_readout", 8 * 256 + 8 * 16),
    ("linoss_readout_bwd_kernel", "surround_readout", 12 * 256 + 8 * 16),
]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("semx_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("kernel,workload,bytes_per_unit", CASES)
def test_profiled_traffic_resolves(bench, kernel, workload, bytes_per_unit):
    traffic, source = bench.profiled_traffic(kernel, workload, UNITS)
    assert source and source.startswith("profiles/")
    assert traffic is not None, f"no traffic_bytes_per_launch entry for {kernel} / {workload}"
    ratio = traffic / (bytes_per_unit * UNITS)
    assert 0.5 < ratio < 2.0, f"{kernel} / {workload}: traffic {ratio:.2f}x algorithmic"
